// Weight-streaming projection kernel of the resident layer path.
//
// Reference arithmetic: the 8x64 fused MAC engine accumulates raw int16 x int16
// products exactly and rounds twice at the end (Q28.20 -> Q16.16 -> Q8.8):
// kernel/mm_stream_8x64_fused_mac.cpp:11-22,89-96,138-205 and
// kernel/compute_core_8x64_unified.cpp:10-39 (golden_projection host:3105-3142).
//
// B200 mapping.  One persistent CTA per SM owns a contiguous slice of the
// weight matrix (whole "units": one output row, or a RoPE / gate-up pair of
// rows).  A producer thread streams the slice through a shared-memory ring
// with 1-D bulk copies (cp.async.bulk, completion on an mbarrier); consumer
// warps own fixed ring stages, read weights and activations with
// 128-bit shared loads and form exact products with the dp2a pipe (weights
// pre-split into unsigned low / signed high bytes, activations packed int16
// pairs), so every MAC is exact and the reduction order is free.  The producer
// starts streaming before the programmatic-dependent-launch wait: weights do
// not depend on the previous kernel, so HBM keeps streaming across kernel
// boundaries.  Each ring wait is bounded; on expiry the kernel records an
// error code in device memory, drains its own copies and returns.
//
// Epilogues fuse what follows the projection in the controller schedule:
// RoPE + KV-cache append (Q/K/V), residual add (O, Down), SiLU(gate) x up
// (Gate/Up), or exact int64 partial sums for the tensor-parallel all-reduce.
#include <cuda_runtime.h>

#include "device_util.cuh"
#include "fixed.cuh"
#include "kernels.cuh"
#include "gemv_common.cuh"

namespace llmx {

// Consumer warps per CTA: up to 16 (latency hiding; the 8-row accumulators fit
// the register budget of 17 warps).
template <int R>
struct Warps {
    static constexpr int kConsumers = 16;
    static constexpr int kThreads = (kConsumers + 1) * 32;  // + one producer warp
};
// Activation prologue (consumer warps): rows -> shared memory, RMS-normalised
// when a norm row is given (stream_rmsnorm kernel/compute_stream.cpp:227-288).
constexpr int kStageBatch = 4;  // 16-byte activation loads in flight per thread while staging

// Rows of a peer all-reduce -> shared memory (raw, before any norm): each
// element waits for every rank's exact sum, x = sat16(resid + round(sum)).
// Block 0 also writes the rows to in.hid_out: they are the residual of the next
// sublayer (the output feature pair of the finished coarse task).
template <int R>
static __device__ void stage_rows_allreduce(const ProjArgs &a, const Step &st, int16_t *xs, int rows, int tid) {
    const int T = blockDim.x - 32, K = a.K;
    const ArInput &in = a.in;
    const uint32_t n = st.ar_base + in.ar_off;
    const int slot = (int)(n & 1u);
    const uint32_t tag = ar_tag(n);
    __shared__ int fail_s;
    if (tid == 0) fail_s = 0;
    consumer_sync();
    for (int i = 4 * tid; i < R * K; i += 4 * T) {  // 4 consecutive elements per step (K % 8 == 0)
        const int r = i / K, e = i - r * K;
        uint2 x = make_uint2(0, 0);
        if (r < rows) {
            int64_t sum[4];
            if (!ar_gather4(in.ar, slot, tag, r, e, &fail_s, sum)) {
                if (!fail_s) atomicCAS(a.error, 0, kErrArTimeout);
                fail_s = 1;
                sum[0] = sum[1] = sum[2] = sum[3] = 0;
            }
            const uint2 rv = *reinterpret_cast<const uint2 *>(in.resid + i);
            const int32_t y0 = sat16(lo16(rv.x) + round_mac(sum[0])), y1 = sat16(hi16(rv.x) + round_mac(sum[1]));
            const int32_t y2 = sat16(lo16(rv.y) + round_mac(sum[2])), y3 = sat16(hi16(rv.y) + round_mac(sum[3]));
            x.x = ((uint32_t)y0 & 0xffffu) | ((uint32_t)y1 << 16);
            x.y = ((uint32_t)y2 & 0xffffu) | ((uint32_t)y3 << 16);
            if (blockIdx.x == 0) *reinterpret_cast<uint2 *>(in.hid_out + i) = x;
        }
        *reinterpret_cast<uint2 *>(xs + i) = x;
    }
    consumer_sync();
}

// Rows of the fused attention + O projection -> shared memory (raw, before any
// norm): x = sat16(resid + round(sum)) from the exact O sums the attention
// kernel added up (the rounding and residual of the O projection's epilogue).
// Block 0 also writes the rows to in.hid_out (the attention sublayer's output).
template <int R>
static __device__ void stage_rows_sums(const ProjArgs &a, int16_t *xs, int rows, int tid) {
    const int T = blockDim.x - 32, K = a.K;
    const ArInput &in = a.in;
    for (int i0 = 4 * tid; i0 < R * K; i0 += 4 * kStageBatch * T) {
        longlong4 sv[kStageBatch];
        uint2 rv[kStageBatch];
#pragma unroll
        for (int k = 0; k < kStageBatch; k++) {  // all loads of a batch in flight first
            const int i = i0 + 4 * k * T;
            if (i < R * K && i / K < rows) {
                sv[k] = *reinterpret_cast<const longlong4 *>(in.sums + i);
                rv[k] = *reinterpret_cast<const uint2 *>(in.resid + i);
            }
        }
#pragma unroll
        for (int k = 0; k < kStageBatch; k++) {
            const int i = i0 + 4 * k * T;
            if (i >= R * K) break;
            uint2 x = make_uint2(0, 0);
            if (i / K < rows) {
                const int32_t y0 = sat16(lo16(rv[k].x) + round_mac(sv[k].x));
                const int32_t y1 = sat16(hi16(rv[k].x) + round_mac(sv[k].y));
                const int32_t y2 = sat16(lo16(rv[k].y) + round_mac(sv[k].z));
                const int32_t y3 = sat16(hi16(rv[k].y) + round_mac(sv[k].w));
                x.x = ((uint32_t)y0 & 0xffffu) | ((uint32_t)y1 << 16);
                x.y = ((uint32_t)y2 & 0xffffu) | ((uint32_t)y3 << 16);
                if (blockIdx.x == 0) *reinterpret_cast<uint2 *>(in.hid_out + i) = x;
            }
            *reinterpret_cast<uint2 *>(xs + i) = x;
        }
    }
    consumer_sync();
}

// In-place RMSNorm of rows already staged in shared memory (all-reduce input);
// red / inv_rms_s: the staging prologue's reduction scratch.
template <int R>
static __device__ void norm_rows_smem(const ProjArgs &a, int16_t *xs, int rows, int tid,
                                      int64_t (*red)[kMaxRows], int32_t *inv_rms_s) {
    const int T = blockDim.x - 32, cw = T / 32;
    const int K = a.K, KV8 = K >> 3;
    if (a.inv_elems == 0) {
        if (tid < R) inv_rms_s[tid] = a.inv_rms_const;
    } else {
        int64_t part[R];
#pragma unroll
        for (int r = 0; r < R; r++) part[r] = 0;
        for (int i = tid; i < K; i += T) {
#pragma unroll
            for (int r = 0; r < R; r++) {
                const int32_t v = xs[r * K + i];
                part[r] += (int64_t)v * v;
            }
        }
#pragma unroll
        for (int r = 0; r < R; r++)
#pragma unroll
            for (int o = 16; o >= 1; o >>= 1) part[r] += shfl_xor64(part[r], o);
        if ((tid & 31) == 0)
#pragma unroll
            for (int r = 0; r < R; r++) red[tid >> 5][r] = part[r];
        consumer_sync();
        if (tid < R) {
            int64_t sum = 0;
            for (int w = 0; w < cw; w++) sum += red[w][tid];
            inv_rms_s[tid] = inv_rms_q88(sum > INT32_MAX ? INT32_MAX : (int32_t)sum, a.inv_elems);
        }
    }
    consumer_sync();
    uint4 *x4 = reinterpret_cast<uint4 *>(xs);
    const uint4 *w4 = reinterpret_cast<const uint4 *>(a.norm);
    for (int i = tid; i < R * KV8; i += T) {
        const int r = i / KV8, v = i - r * KV8;
        const uint4 xv = x4[i], wv = w4[v];
        const int64_t inv = r < rows ? inv_rms_s[r] : 0;
        const uint32_t xw[4] = {xv.x, xv.y, xv.z, xv.w};
        const uint32_t ww[4] = {wv.x, wv.y, wv.z, wv.w};
        uint32_t ow[4];
#pragma unroll
        for (int q = 0; q < 4; q++) {
            const int32_t y0 = sat16(rnd((int64_t)lo16(xw[q]) * inv * lo16(ww[q]), 16));
            const int32_t y1 = sat16(rnd((int64_t)hi16(xw[q]) * inv * hi16(ww[q]), 16));
            ow[q] = ((uint32_t)y0 & 0xffffu) | ((uint32_t)y1 << 16);
        }
        x4[i] = make_uint4(ow[0], ow[1], ow[2], ow[3]);
    }
    consumer_sync();
}

template <int R>
static __device__ void stage_rows(const ProjArgs &a, const Step &st, int16_t *xs, int rows, int tid) {
    constexpr int CW = Warps<R>::kConsumers;  // upper bound of the consumer warps
    const int T = blockDim.x - 32, cw = T / 32;
    const int K = a.K, KV8 = K >> 3;
    __shared__ int32_t inv_rms_s[kMaxRows];
    __shared__ int64_t red[CW][kMaxRows];
    if (a.in.ar.n > 1) {  // tensor parallel: the previous projection's all-reduce, finished here
        stage_rows_allreduce<R>(a, st, xs, rows, tid);
        if (a.norm != nullptr) norm_rows_smem<R>(a, xs, rows, tid, red, inv_rms_s);
        return;
    }
    if (a.in.sums != nullptr) {  // the fused attention's O sums, finished here
        stage_rows_sums<R>(a, xs, rows, tid);
        if (a.norm != nullptr) norm_rows_smem<R>(a, xs, rows, tid, red, inv_rms_s);
        return;
    }
    if (a.norm != nullptr) {
        if (a.inv_elems == 0) {
            // recip(fm(K)) == 0: mean == 0 for every input, inv_rms is a constant
            if (tid < R) inv_rms_s[tid] = a.inv_rms_const;
        } else {
            int64_t part[R];
#pragma unroll
            for (int r = 0; r < R; r++) part[r] = 0;
            for (int i = tid; i < K; i += T) {
#pragma unroll
                for (int r = 0; r < R; r++)
                    if (r < rows) {
                        const int32_t v = a.x[(size_t)r * K + i];
                        part[r] += (int64_t)v * v;
                    }
            }
#pragma unroll
            for (int r = 0; r < R; r++)
#pragma unroll
                for (int o = 16; o >= 1; o >>= 1) part[r] += shfl_xor64(part[r], o);
            if ((tid & 31) == 0)
#pragma unroll
                for (int r = 0; r < R; r++) red[tid >> 5][r] = part[r];
            consumer_sync();
            if (tid < R) {
                int64_t sum = 0;
                for (int w = 0; w < cw; w++) sum += red[w][tid];
                // saturating running sum == min(total, INT32_MAX): every term is >= 0
                inv_rms_s[tid] = inv_rms_q88(sum > INT32_MAX ? INT32_MAX : (int32_t)sum, a.inv_elems);
            }
        }
        consumer_sync();
        const uint4 *x4 = reinterpret_cast<const uint4 *>(a.x);
        const uint4 *w4 = reinterpret_cast<const uint4 *>(a.norm);
        // all loads of a batch in flight before any is used (one L2 round trip per batch)
        for (int i0 = tid; i0 < R * KV8; i0 += kStageBatch * T) {
            uint4 xv[kStageBatch], wv[kStageBatch];
#pragma unroll
            for (int k = 0; k < kStageBatch; k++) {
                const int i = i0 + k * T, r = i / KV8, v = i - r * KV8;
                xv[k] = wv[k] = make_uint4(0, 0, 0, 0);
                if (i < R * KV8 && r < rows) {
                    xv[k] = x4[(size_t)r * KV8 + v];
                    wv[k] = w4[v];
                }
            }
#pragma unroll
            for (int k = 0; k < kStageBatch; k++) {
                const int i = i0 + k * T, r = i / KV8;
                if (i >= R * KV8) break;
                const int64_t inv = r < rows ? inv_rms_s[r] : 0;
                const uint32_t xw[4] = {xv[k].x, xv[k].y, xv[k].z, xv[k].w};
                const uint32_t ww[4] = {wv[k].x, wv[k].y, wv[k].z, wv[k].w};
                uint32_t ow[4];
#pragma unroll
                for (int q = 0; q < 4; q++) {
                    const int32_t y0 = sat16(rnd((int64_t)lo16(xw[q]) * inv * lo16(ww[q]), 16));
                    const int32_t y1 = sat16(rnd((int64_t)hi16(xw[q]) * inv * hi16(ww[q]), 16));
                    ow[q] = ((uint32_t)y0 & 0xffffu) | ((uint32_t)y1 << 16);
                }
                reinterpret_cast<uint4 *>(xs)[i] = make_uint4(ow[0], ow[1], ow[2], ow[3]);
            }
        }
    } else {
        const uint4 *x4 = reinterpret_cast<const uint4 *>(a.x);
        for (int i0 = tid; i0 < R * KV8; i0 += kStageBatch * T) {
            uint4 xv[kStageBatch];
#pragma unroll
            for (int k = 0; k < kStageBatch; k++) {
                const int i = i0 + k * T;
                xv[k] = (i < R * KV8 && i / KV8 < rows) ? x4[i] : make_uint4(0, 0, 0, 0);
            }
#pragma unroll
            for (int k = 0; k < kStageBatch; k++) {
                const int i = i0 + k * T;
                if (i < R * KV8) reinterpret_cast<uint4 *>(xs)[i] = xv[k];
            }
        }
    }
    consumer_sync();
}

template <int R, int EPI>
struct GemvTraits {
    static constexpr int U = (EPI == EPI_QKV || EPI == EPI_SILU) ? 2 : 1;  // rows per unit
};

// unit -> this CTA's contiguous range [u0, u1)
static __device__ __forceinline__ void unit_range(int nunits, int &u0, int &u1) {
    u0 = (int)((int64_t)nunits * blockIdx.x / gridDim.x);
    u1 = (int)((int64_t)nunits * (blockIdx.x + 1) / gridDim.x);
}

template <int R, int EPI, int VPL, int P>
__global__ void __launch_bounds__(Warps<R>::kThreads, 1) k_gemv(const ProjArgs a) {
    LLMX_TL_GUARD(a.tl_slot);
    constexpr int U = GemvTraits<R, EPI>::U;
    constexpr int N = U * R;  // int64 sums per unit
    extern __shared__ __align__(128) char smem[];
    const int K = a.K, KV8 = K >> 3;
    const int unit_words = U * (K >> 1);
    const uint32_t unit_bytes = (uint32_t)unit_words * 4;
    // G stages, each holding one chunk of B consecutive units (one bulk copy);
    // consumer warp w = (g*B + b)*P + p belongs to group g, which owns stage g,
    // and takes part p of unit b of every chunk j = g, g+G, g+2G, ...  Every
    // stage is thus waited on by the same warps, in phase order.
    const int G = a.stages, B = a.units_per_chunk, C = G * B * P;
    const int S = G;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem);
    uint64_t *empty = full + kMaxStages;
    char *ring = smem + 2 * kMaxStages * sizeof(uint64_t);
    const uint32_t chunk_bytes = unit_bytes * (uint32_t)B;
    int16_t *xs = reinterpret_cast<int16_t *>(ring + (size_t)S * chunk_bytes);
    // P > 1: per (round parity, unit slot) int64 sums of the P parts and arrival
    // counters; the last part to arrive runs the epilogue and clears the slot.
    int64_t *cacc = reinterpret_cast<int64_t *>(xs + (size_t)R * K);
    int32_t *ccnt = reinterpret_cast<int32_t *>(cacc + 2 * G * B * N);
    if (P > 1) {
        for (int i = threadIdx.x; i < 2 * G * B * N; i += blockDim.x) cacc[i] = 0;
        for (int i = threadIdx.x; i < 2 * G * B; i += blockDim.x) ccnt[i] = 0;
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nunits = a.npairs * 2 / U;
    int u0, u1;
    unit_range(nunits, u0, u1);
    const int nloc = u1 - u0;
    const int nchunks = (nloc + B - 1) / B;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; s++) {
            mbar_init(full + s, 1);
            mbar_init(empty + s, (uint32_t)(B * P));  // every warp of the owning group arrives
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();

    if (warp == (int)(blockDim.x >> 5) - 1) {  // ---------------- producer warp -------------
        if (lane == 0) {
            const uint64_t policy = evict_first_policy();  // weights are read once per step
            const char *src = reinterpret_cast<const char *>(a.w) + (size_t)u0 * unit_bytes;
            bool ok = true;
            int issued = 0;
            for (int j = 0; j < nchunks; j++) {
                const int s = j % S;
                if (j >= S && !mbar_wait(empty + s, ((j / S) - 1) & 1)) {
                    ok = false;
                    break;
                }
                const uint32_t bytes = (uint32_t)min(B, nloc - j * B) * unit_bytes;
                mbar_expect_tx(full + s, bytes);
                bulk_g2s_hint(ring + (size_t)s * chunk_bytes, src + (size_t)j * chunk_bytes, bytes, full + s, policy);
                issued = j + 1;
                if (j == S - 1) pdl_wait();  // ring primed before waiting on the producer kernel
            }
            if (nchunks < S) pdl_wait();
            if (!ok) {
                atomicExch(a.error, 1);
                // drain: wait (bounded) for the last fill of every stage this thread issued
                for (int s = 0; s < S && s < issued; s++) {
                    const int last = s + ((issued - 1 - s) / S) * S;
                    (void)mbar_wait(full + s, (last / S) & 1);
                }
            }
        }
        return;
    }

    // ---------------- consumer warps ----------------------------------------
    const int tid = threadIdx.x;
    const Step st = load_step(a.step);
    pdl_wait();
    pdl_trigger();
    if (a.zero != nullptr)  // the previous kernel has read these sums: clear them for their next use
        for (int i = blockIdx.x * (blockDim.x - 32) + tid; i < a.zero_n; i += gridDim.x * (blockDim.x - 32))
            a.zero[i] = 0;
    const int rows = st.rows - a.row0;  // rows of this launch (a block may be split in row groups)
    const uint32_t ar_n = st.ar_base + a.ar_off;  // EPI_PARTIAL: this projection's all-reduce
    stage_rows<R>(a, st, xs, rows, tid);
    const uint4 *xs4 = reinterpret_cast<const uint4 *>(xs);
    uint4 xr[8];  // 1-row decode with K <= 2048: this lane's activation vectors stay in registers
    if (R == 1 && VPL > 0 && VPL <= 8) {
#pragma unroll
        for (int k = 0; k < 8; k++)
            if (k < VPL) xr[k] = xs4[k * 32 + lane];
    }

    // A parity wait is only unambiguous for the phase right after the one the
    // waiter consumed last, so each group waits on its own stage chunk by chunk.
    const int grp = warp / (B * P), within = warp - grp * (B * P);
    const int slot = within / P, part = within - slot * P;
    for (int j = grp; warp < C && j < nchunks; j += G) {
        const int s = j % S;
        if (!__all_sync(0xffffffffu, mbar_wait(full + s, (j / S) & 1))) {  // warp-uniform decision
            if (lane == 0) atomicExch(a.error, 2);
            break;
        }
        const int jl = j * B + slot;  // local unit index
        int64_t acc[N];
        if (jl < nloc)
            unit_dots<R, U, VPL, P>(
                reinterpret_cast<const uint4 *>(ring + (size_t)s * chunk_bytes + (size_t)slot * unit_bytes), xs4, xr,
                KV8, lane, part, acc);
        __syncwarp();
        if (lane == 0) mbar_arrive(empty + s);  // this warp's part of the stage is free
        if (jl >= nloc) continue;

        int idx;
        int64_t tot = warp_reduce_n<N>(acc, lane, idx);
        if constexpr (P > 1) {
            // Lock-free combine: no warp ever waits for another part.
            const int cs = ((j / G) & 1) * G * B + grp * B + slot;
            int64_t *cb = cacc + (size_t)cs * N;
            if ((lane & (32 / N - 1)) == 0)
                atomicAdd(reinterpret_cast<unsigned long long *>(cb + idx), (unsigned long long)tot);
            __threadfence_block();
            __syncwarp();
            int last = 0;
            if (lane == 0) last = atomicAdd(ccnt + cs, 1) == P - 1;
            if (!__shfl_sync(0xffffffffu, last, 0)) continue;
            __threadfence_block();
            tot = *reinterpret_cast<volatile int64_t *>(cb + idx);
            __syncwarp();
            // reused two rounds later, after this warp has released the next chunk
            if ((lane & (32 / N - 1)) == 0) cb[idx] = 0;
            if (lane == 0) ccnt[cs] = 0;
        }
        const int unit = u0 + jl;
        if (U == 2) {
            constexpr int kPartnerBit = 32 / N;
            const int64_t other = __shfl_sync(0xffffffffu, tot, lane | kPartnerBit);
            const int r = idx >> 1;
            if ((lane & (kPartnerBit - 1)) != 0 || (idx & 1) != 0 || r >= rows) continue;
            const int32_t y0 = round_mac(tot), y1 = round_mac(other);
            if (EPI == EPI_SILU) {
                a.out[(size_t)r * a.out_stride + unit] = (int16_t)silu_mul(y0, y1, a.etab);
            } else {  // EPI_QKV: unit = pair (i, i + hd/2) of a head
                const int half = a.hd >> 1;
                const int pos = st.position + r;
                int pp = unit;
                if (pp < a.q_pairs + a.kv_pairs) {
                    // RoPE rotate_fix16_pair_with_quantized_rope host:4765-4788
                    const bool isq = pp < a.q_pairs;
                    if (!isq) pp -= a.q_pairs;
                    const int head = pp / half, i = pp - head * half;
                    const int64_t cs = a.rope[(size_t)pos * a.hd + i];
                    const int64_t sn = a.rope[(size_t)pos * a.hd + half + i];
                    const int16_t z0 = (int16_t)sat16(rnd((int64_t)y0 * cs - (int64_t)y1 * sn, 8));
                    const int16_t z1 = (int16_t)sat16(rnd((int64_t)y1 * cs + (int64_t)y0 * sn, 8));
                    int16_t *dst = isq ? a.out + (size_t)r * a.out_stride + (size_t)head * a.hd
                                       : a.kc + ((size_t)head * a.max_seq + pos) * a.hd;
                    dst[i] = z0;
                    dst[i + half] = z1;
                } else {
                    pp -= a.q_pairs + a.kv_pairs;
                    const int head = pp / half, i = pp - head * half;
                    int16_t *dst = a.vc + ((size_t)head * a.max_seq + pos) * a.hd;
                    dst[i] = (int16_t)y0;
                    dst[i + half] = (int16_t)y1;
                }
            }
        } else {
            const int r = idx;
            if ((lane & (32 / N - 1)) != 0 || r >= rows) continue;
            if (EPI == EPI_PARTIAL) {
                if (a.ar.n > 1) {  // straight into every rank's exchange region (NVLink stores)
                    const size_t w = ar_word_index((int)(ar_n & 1u), a.ar.me, r, a.ar.hidden, unit);
                    const uint64_t word = ar_pack(tot, ar_tag(ar_n));
                    for (int p = 0; p < a.ar.n; p++)
                        ar_store(reinterpret_cast<uint64_t *>(a.ar.base[p] + kArHeader) + w, word);
                } else {
                    a.partial[(size_t)r * a.out_stride + unit] = tot;
                }
            } else {  // EPI_RESID
                const size_t o = (size_t)r * a.out_stride + unit;
                a.out[o] = (int16_t)sat16((int32_t)a.resid[o] + round_mac(tot));
            }
        }
    }
}

size_t gemv_smem_bytes(int rows_tmpl, int epi, int K, int stages, int units_per_chunk, int parts) {
    const int U = (epi == EPI_QKV || epi == EPI_SILU) ? 2 : 1;
    const size_t combine = parts > 1 ? (size_t)2 * stages * units_per_chunk * (U * rows_tmpl * 8 + 4) : 0;
    return 2 * kMaxStages * sizeof(uint64_t) + (size_t)stages * units_per_chunk * U * K * 2 +
           (size_t)rows_tmpl * K * 2 + combine;
}

// Ring plan.  1-D bulk copies only stream at full HBM rate when each copy is
// large (>= 16 KiB on B200: 8 KiB copies cap near 4 TB/s), so a stage holds B
// consecutive units making a ~32 KiB chunk, and G stages form the ring; the
// consumer warps are G groups of B.  A unit of 16 KiB or more (the FFN-wide
// Down rows) fills a stage alone and would leave one warp per stage to digest
// it, so such units are split over P = 4 (or, for a deeper ring, 2) warps.  Limits: G*B*P <= consumer
// warps of the kernel, G >= 2 (double buffering), shared memory within max_smem.
int gemv_stages(int rows_tmpl, int epi, int K, int max_smem, int ring_bytes, int *units_per_chunk, int *parts,
                int max_warps) {
    const int U = (epi == EPI_QKV || epi == EPI_SILU) ? 2 : 1;
    const int unit = U * K * 2;
    const int cmax = max_warps < 2 ? 2 : (max_warps > 16 ? 16 : max_warps);  // consumer warps
    int B = (32 * 1024) / unit;
    if (B < 1) B = 1;
    if (B > cmax / 2) B = cmax / 2;
    int P = 1;
    if (U == 1 && B == 1 && unit >= 16 * 1024) {
        // stages first (what the ring and shared memory allow), then as many
        // warps per unit as the stages leave
        int g0 = ring_bytes / unit;
        if (g0 < 2) g0 = 2;
        while (g0 > 2 && gemv_smem_bytes(rows_tmpl, epi, K, g0, 1, 4) > (size_t)max_smem) g0--;
        P = cmax / g0 >= 4 ? 4 : (cmax / g0 >= 2 ? 2 : 1);
    }
    int G = ring_bytes / (B * unit);
    if (G > cmax / (B * P)) G = cmax / (B * P);
    if (G < 2) G = 2;
    while (G > 1 && gemv_smem_bytes(rows_tmpl, epi, K, G, B, P) > (size_t)max_smem) G--;
    while (B > 1 && gemv_smem_bytes(rows_tmpl, epi, K, G, B, P) > (size_t)max_smem) B--;
    *units_per_chunk = B;
    *parts = P;
    return G;
}

template <int R, int EPI, int VPL, int P>
static cudaError_t launch_gemv_v(const ProjArgs &a, int grid, cudaStream_t st) {
    ProjArgs c = a;
    LLMX_TL_TAKE(c, EPI == EPI_QKV ? "gemv/qkv" : EPI == EPI_RESID ? "gemv/resid" : EPI == EPI_SILU ? "gemv/gate_up" : "gemv/partial");
    void *args[] = {&c};
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3((a.stages * a.units_per_chunk * P + 1) * 32);  // consumer groups + producer
    cfg.dynamicSmemBytes = gemv_smem_bytes(R, EPI, a.K, a.stages, a.units_per_chunk, P);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelExC(&cfg, (const void *)k_gemv<R, EPI, VPL, P>, args);
}

// Fully unrolled paths for the Qwen2.5-3B input widths: K = 2048 (hidden) and
// K = 11008 (FFN, single GPU); everything else takes the generic loop.
// Units split over 4 warps exist only for the one-row-per-unit epilogues.
template <int R, int EPI>
static cudaError_t launch_gemv_t(const ProjArgs &a, int grid, cudaStream_t st) {
    constexpr bool kSplit = EPI == EPI_RESID || EPI == EPI_PARTIAL;
    if constexpr (kSplit) {
        if (a.parts == 4) {
            if constexpr (R <= 2)
                if (a.K == 11008) return launch_gemv_v<R, EPI, 43, 4>(a, grid, st);
            return launch_gemv_v<R, EPI, 0, 4>(a, grid, st);
        }
        if (a.parts == 2) {
            if constexpr (R <= 2)
                if (a.K == 11008) return launch_gemv_v<R, EPI, 43, 2>(a, grid, st);
            return launch_gemv_v<R, EPI, 0, 2>(a, grid, st);
        }
        if constexpr (R <= 2)
            if (a.K == 11008 && a.parts == 1) return launch_gemv_v<R, EPI, 43, 1>(a, grid, st);
    }
    if (a.parts != 1) return cudaErrorInvalidValue;
    if (a.K == 2048) return launch_gemv_v<R, EPI, 8, 1>(a, grid, st);
    return launch_gemv_v<R, EPI, 0, 1>(a, grid, st);
}

template <int EPI>
static cudaError_t launch_gemv_r(const ProjArgs &a, int rows_tmpl, int grid, cudaStream_t s) {
    switch (rows_tmpl) {
    case 1: return launch_gemv_t<1, EPI>(a, grid, s);
    case 2: return launch_gemv_t<2, EPI>(a, grid, s);
    case 4: return launch_gemv_t<4, EPI>(a, grid, s);
    default: return launch_gemv_t<8, EPI>(a, grid, s);
    }
}

cudaError_t launch_proj(const ProjArgs &a, int epi, int rows_tmpl, int grid, cudaStream_t s) {
    switch (epi) {
    case EPI_QKV: return launch_gemv_r<EPI_QKV>(a, rows_tmpl, grid, s);
    case EPI_RESID: return launch_gemv_r<EPI_RESID>(a, rows_tmpl, grid, s);
    case EPI_SILU: return launch_gemv_r<EPI_SILU>(a, rows_tmpl, grid, s);
    default: return launch_gemv_r<EPI_PARTIAL>(a, rows_tmpl, grid, s);
    }
}

// Dynamic shared memory limit and, when carveout >= 0, the preferred shared
// memory carveout (percent of the SM's unified L1 / shared storage) of one
// instantiation.
template <int R, int EPI, int VPL, int P>
static cudaError_t configure_v(int bytes, int carveout) {
    cudaError_t e = cudaFuncSetAttribute(k_gemv<R, EPI, VPL, P>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e == cudaSuccess && carveout >= 0)
        e = cudaFuncSetAttribute(k_gemv<R, EPI, VPL, P>, cudaFuncAttributePreferredSharedMemoryCarveout, carveout);
    return e;
}

template <int R, int EPI>
static cudaError_t configure_r(int bytes, int carveout) {
    cudaError_t e = configure_v<R, EPI, 8, 1>(bytes, carveout);
    if (e) return e;
    if constexpr (EPI == EPI_RESID || EPI == EPI_PARTIAL) {
        if (R <= 2) {
            if ((e = configure_v<R, EPI, 43, 1>(bytes, carveout))) return e;
            if ((e = configure_v<R, EPI, 43, 4>(bytes, carveout))) return e;
            if ((e = configure_v<R, EPI, 43, 2>(bytes, carveout))) return e;
        }
        if ((e = configure_v<R, EPI, 0, 4>(bytes, carveout))) return e;
        if ((e = configure_v<R, EPI, 0, 2>(bytes, carveout))) return e;
    }
    return configure_v<R, EPI, 0, 1>(bytes, carveout);
}

template <int EPI>
static cudaError_t configure_epi(int bytes, int carveout) {
    cudaError_t e;
    if ((e = configure_r<1, EPI>(bytes, carveout))) return e;
    if ((e = configure_r<2, EPI>(bytes, carveout))) return e;
    if ((e = configure_r<4, EPI>(bytes, carveout))) return e;
    return configure_r<8, EPI>(bytes, carveout);
}

cudaError_t proj_configure(int max_smem_bytes, int carveout) {
    cudaError_t e;
    if ((e = configure_epi<EPI_QKV>(max_smem_bytes, carveout))) return e;
    if ((e = configure_epi<EPI_RESID>(max_smem_bytes, carveout))) return e;
    if ((e = configure_epi<EPI_SILU>(max_smem_bytes, carveout))) return e;
    return configure_epi<EPI_PARTIAL>(max_smem_bytes, carveout);
}

}  // namespace llmx

LLMX_TL_READER(gemv)
