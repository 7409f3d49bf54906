// sm_100a kernels of the resident decoder-layer path (Task 18 / 19 / 20).
//
// Projections (kernel/mm_stream_8x64_fused_mac.cpp:138-205 + the conversion of
// kernel/compute_core_8x64_unified.cpp:10-39) become one weight-streaming
// kernel: each warp owns a pair of output rows, streams both rows once from HBM
// with 128-bit loads and forms exact int16 x int16 dot products with the
// integer dp2a pipe (weights pre-split into signed high / unsigned low bytes,
// activations packed as int16 pairs), so every MAC is exact and reduction order
// is free.  The rounding epilogue of the MAC engine is fused with what follows
// the projection in the controller's schedule: RoPE + KV append (Q/K/V),
// residual add (O, Down), SiLU x Up (Gate/Up), or an int64 export for the
// tensor-parallel all-reduce.  RMSNorm (kernel/compute_stream.cpp:227-288) is
// the prologue that stages the activations in shared memory.
//
// Attention lives in attention.cu.
#include <cuda_runtime.h>

#include "device_util.cuh"
#include "fixed.cuh"
#include "kernels.cuh"

namespace llmx {

// golden_silu host:658-668 / cu_silu_approx kernel/compute_stream.cpp:88-96,
// then x up with one rounding (stream_silu_mul :123-164).
__device__ __forceinline__ int32_t silu_mul(int32_t g, int32_t u, const int16_t *__restrict__ etab) {
    int32_t s;
    if (g >= 0) {
        const int32_t idx = -g < -2048 ? 0 : 2048 - g;
        const int32_t e = __ldg(etab + idx);
        const int32_t r = recip_q88(sat16(256 + e));
        s = sat16(rnd((int64_t)g * r, 8));
    } else {
        const int32_t idx = g < -2048 ? 0 : g + 2048;
        const int32_t e = __ldg(etab + idx);
        const int32_t r = recip_q88(sat16(256 + e));
        s = sat16(rnd((int64_t)g * e * r, 16));
    }
    return sat16(rnd((int64_t)s * u, 8));
}

// Halving ("transpose") warp reduction of N int64 values: afterwards lane L
// holds the warp total of value index idx(L); lanes differing only in bits
// below 32/N hold the same index.  N <= 16.
template <int N>
__device__ __forceinline__ int64_t warp_reduce_n(int64_t (&v)[N], int lane, int &idx) {
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

// --------------------------------------------------------------------------
// activation prologue: rows -> shared memory (optionally RMS-normalised)
// --------------------------------------------------------------------------
template <int R>
__device__ void stage_rows(const ProjArgs &a, int16_t *xs, int rows) {
    const int K = a.K;
    const int KV8 = K >> 3;
    uint4 *xs4 = reinterpret_cast<uint4 *>(xs);
    const uint4 *x4 = reinterpret_cast<const uint4 *>(a.x);
    __shared__ int32_t inv_rms_s[kMaxRows];
    if (a.norm != nullptr) {
        if (a.inv_elems == 0) {
            // recip(fm(K)) == 0: mean == 0 for every input, inv_rms is a constant.
            if (threadIdx.x < R) inv_rms_s[threadIdx.x] = a.inv_rms_const;
        } else {
            __shared__ int64_t red[kWarps][kMaxRows];
            int64_t part[R];
#pragma unroll
            for (int r = 0; r < R; r++) part[r] = 0;
            for (int i = threadIdx.x; i < K; i += blockDim.x) {
#pragma unroll
                for (int r = 0; r < R; r++) {
                    if (r < rows) {
                        const int32_t v = a.x[(size_t)r * K + i];
                        part[r] += (int64_t)v * v;
                    }
                }
            }
#pragma unroll
            for (int r = 0; r < R; r++) {
#pragma unroll
                for (int o = 16; o >= 1; o >>= 1) part[r] += shfl_xor64(part[r], o);
            }
            const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
            if (lane == 0) {
#pragma unroll
                for (int r = 0; r < R; r++) red[warp][r] = part[r];
            }
            __syncthreads();
            if (threadIdx.x < R) {
                int64_t s = 0;
                for (int w = 0; w < (int)(blockDim.x >> 5); w++) s += red[w][threadIdx.x];
                // saturating running sum == min(total, INT32_MAX) since terms are >= 0
                const int32_t sum = s > INT32_MAX ? INT32_MAX : (int32_t)s;
                inv_rms_s[threadIdx.x] = inv_rms_q88(sum, a.inv_elems);
            }
        }
        __syncthreads();
        for (int i = threadIdx.x; i < R * K; i += blockDim.x) {
            const int r = i / K, e = i - r * K;
            int32_t y = 0;
            if (r < rows) {
                const int64_t p = (int64_t)a.x[(size_t)r * K + e] * inv_rms_s[r] * a.norm[e];
                y = sat16(rnd(p, 16));
            }
            xs[i] = (int16_t)y;
        }
    } else {
        for (int i = threadIdx.x; i < R * KV8; i += blockDim.x) {
            const int r = i / KV8;
            xs4[i] = r < rows ? x4[i] : make_uint4(0, 0, 0, 0);
        }
    }
    __syncthreads();
}

// --------------------------------------------------------------------------
// projection kernel
// --------------------------------------------------------------------------
template <int R, int EPI>
__global__ void __launch_bounds__(kWarps * 32) k_proj(const ProjArgs a) {
    extern __shared__ __align__(16) int16_t xs[];
    constexpr int N = 2 * R;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int K = a.K, KV8 = K >> 3;
    const int nchunks = (KV8 + 255) >> 8;
    const int nw = gridDim.x * kWarps;
    int p = blockIdx.x * kWarps + warp;

    uint4 wa[8], wb[8];
    auto load_chunk = [&](int pair, int c) {
        const uint4 *base = reinterpret_cast<const uint4 *>(a.w + (size_t)pair * K);
#pragma unroll
        for (int j = 0; j < 8; j++) {
            const int v = (c << 8) + (j << 5) + lane;
            if (v < KV8) {
                wa[j] = ld_stream(base + v);
                wb[j] = ld_stream(base + KV8 + v);
            } else {
                wa[j] = make_uint4(0, 0, 0, 0);
                wb[j] = make_uint4(0, 0, 0, 0);
            }
        }
    };

    // Weights do not depend on the producer kernel: start streaming them
    // before waiting for it (programmatic dependent launch).
    bool preloaded = p < a.npairs;
    if (preloaded) load_chunk(p, 0);
    pdl_wait();
    pdl_trigger();
    const Step st = *a.step;
    const int rows = st.rows;
    stage_rows<R>(a, xs, rows);
    const uint4 *xs4 = reinterpret_cast<const uint4 *>(xs);

    for (; p < a.npairs; p += nw) {
        int64_t acc[N];
#pragma unroll
        for (int i = 0; i < N; i++) acc[i] = 0;
        for (int c = 0; c < nchunks; c++) {
            if (c > 0 || !preloaded) load_chunk(p, c);
            int lo[N], hi[N];
#pragma unroll
            for (int i = 0; i < N; i++) lo[i] = hi[i] = 0;
#pragma unroll
            for (int j = 0; j < 8; j++) {
                const int v = (c << 8) + (j << 5) + lane;
                if (v < KV8) {
#pragma unroll
                    for (int r = 0; r < R; r++) {
                        const uint4 x = xs4[r * KV8 + v];
                        lo[2 * r] = dp2a_lo_su(x.x, wa[j].x, lo[2 * r]);
                        hi[2 * r] = dp2a_hi_ss(x.x, wa[j].x, hi[2 * r]);
                        lo[2 * r] = dp2a_lo_su(x.y, wa[j].y, lo[2 * r]);
                        hi[2 * r] = dp2a_hi_ss(x.y, wa[j].y, hi[2 * r]);
                        lo[2 * r] = dp2a_lo_su(x.z, wa[j].z, lo[2 * r]);
                        hi[2 * r] = dp2a_hi_ss(x.z, wa[j].z, hi[2 * r]);
                        lo[2 * r] = dp2a_lo_su(x.w, wa[j].w, lo[2 * r]);
                        hi[2 * r] = dp2a_hi_ss(x.w, wa[j].w, hi[2 * r]);
                        lo[2 * r + 1] = dp2a_lo_su(x.x, wb[j].x, lo[2 * r + 1]);
                        hi[2 * r + 1] = dp2a_hi_ss(x.x, wb[j].x, hi[2 * r + 1]);
                        lo[2 * r + 1] = dp2a_lo_su(x.y, wb[j].y, lo[2 * r + 1]);
                        hi[2 * r + 1] = dp2a_hi_ss(x.y, wb[j].y, hi[2 * r + 1]);
                        lo[2 * r + 1] = dp2a_lo_su(x.z, wb[j].z, lo[2 * r + 1]);
                        hi[2 * r + 1] = dp2a_hi_ss(x.z, wb[j].z, hi[2 * r + 1]);
                        lo[2 * r + 1] = dp2a_lo_su(x.w, wb[j].w, lo[2 * r + 1]);
                        hi[2 * r + 1] = dp2a_hi_ss(x.w, wb[j].w, hi[2 * r + 1]);
                    }
                }
            }
            // |lo| <= 32 * 2 * 255 * 32768 < 2^29, |hi| <= 32 * 2 * 128 * 32768 = 2^28
#pragma unroll
            for (int i = 0; i < N; i++) acc[i] += (int64_t)hi[i] * 256 + lo[i];
        }
        const int pcur = p;
        // start streaming the next pair before the reduction and epilogue
        preloaded = p + nw < a.npairs;
        if (preloaded) load_chunk(p + nw, 0);

        int idx;
        const int64_t tot = warp_reduce_n<N>(acc, lane, idx);
        constexpr int kPartnerBit = 32 / N;
        const int64_t other = __shfl_sync(0xffffffffu, tot, lane | kPartnerBit);
        const int r = idx >> 1;
        if ((lane & (kPartnerBit - 1)) != 0 || (idx & 1) != 0 || r >= rows) continue;
        if (EPI == EPI_PARTIAL) {
            a.partial[(size_t)r * (2 * a.npairs) + 2 * pcur] = tot;
            a.partial[(size_t)r * (2 * a.npairs) + 2 * pcur + 1] = other;
            continue;
        }
        const int32_t y0 = round_mac(tot), y1 = round_mac(other);
        if (EPI == EPI_RESID) {
            const size_t o = (size_t)r * a.out_stride + 2 * pcur;
            a.out[o] = (int16_t)sat16((int32_t)a.resid[o] + y0);
            a.out[o + 1] = (int16_t)sat16((int32_t)a.resid[o + 1] + y1);
        } else if (EPI == EPI_SILU) {
            a.out[(size_t)r * a.out_stride + pcur] = (int16_t)silu_mul(y0, y1, a.etab);
        } else if (EPI == EPI_QKV) {
            const int half = a.hd >> 1;
            const int pos = st.position + r;
            int pp = pcur;
            if (pp < a.q_pairs + a.kv_pairs) {
                // RoPE rotate_fix16_pair_with_quantized_rope host:4765-4788
                const bool isq = pp < a.q_pairs;
                if (!isq) pp -= a.q_pairs;
                const int head = pp / half, i = pp - head * half;
                const int64_t c = a.rope[(size_t)pos * a.hd + i];
                const int64_t s = a.rope[(size_t)pos * a.hd + half + i];
                const int16_t z0 = (int16_t)sat16(rnd((int64_t)y0 * c - (int64_t)y1 * s, 8));
                const int16_t z1 = (int16_t)sat16(rnd((int64_t)y1 * c + (int64_t)y0 * s, 8));
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
    }
}

template <int R, int EPI>
static cudaError_t launch_proj_t(const ProjArgs &a, int grid, cudaStream_t s) {
    const size_t smem = (size_t)R * a.K * sizeof(int16_t);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kWarps * 32);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, k_proj<R, EPI>, a);
}

template <int EPI>
static cudaError_t launch_proj_r(const ProjArgs &a, int rows_tmpl, int grid, cudaStream_t s) {
    switch (rows_tmpl) {
    case 1: return launch_proj_t<1, EPI>(a, grid, s);
    case 2: return launch_proj_t<2, EPI>(a, grid, s);
    case 4: return launch_proj_t<4, EPI>(a, grid, s);
    default: return launch_proj_t<8, EPI>(a, grid, s);
    }
}

cudaError_t launch_proj(const ProjArgs &a, int epi, int rows_tmpl, int grid, cudaStream_t s) {
    switch (epi) {
    case EPI_QKV: return launch_proj_r<EPI_QKV>(a, rows_tmpl, grid, s);
    case EPI_RESID: return launch_proj_r<EPI_RESID>(a, rows_tmpl, grid, s);
    case EPI_SILU: return launch_proj_r<EPI_SILU>(a, rows_tmpl, grid, s);
    default: return launch_proj_r<EPI_PARTIAL>(a, rows_tmpl, grid, s);
    }
}

size_t proj_smem_bytes(int rows_tmpl, int K) { return (size_t)rows_tmpl * K * sizeof(int16_t); }

template <int EPI>
static cudaError_t configure_epi(int bytes) {
    cudaError_t e;
    if ((e = cudaFuncSetAttribute(k_proj<1, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes))) return e;
    if ((e = cudaFuncSetAttribute(k_proj<2, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes))) return e;
    if ((e = cudaFuncSetAttribute(k_proj<4, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes))) return e;
    return cudaFuncSetAttribute(k_proj<8, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
}

// Opt every projection instantiation into large dynamic shared memory on the
// current device (8 rows x 11008 inputs = 172 KiB for the Down projection).
cudaError_t proj_configure(int max_smem_bytes) {
    cudaError_t e;
    if ((e = configure_epi<EPI_QKV>(max_smem_bytes))) return e;
    if ((e = configure_epi<EPI_RESID>(max_smem_bytes))) return e;
    if ((e = configure_epi<EPI_SILU>(max_smem_bytes))) return e;
    return configure_epi<EPI_PARTIAL>(max_smem_bytes);
}

template <int R, int EPI>
static int occ_t(int K) {
    int n = 0;
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, k_proj<R, EPI>, kWarps * 32,
                                                  (size_t)R * K * sizeof(int16_t));
    return n;
}
int proj_max_ctas_per_sm(int epi, int rows_tmpl, int K) {
    // all epilogues share the register/smem profile closely enough; use RESID
    (void)epi;
    switch (rows_tmpl) {
    case 1: return occ_t<1, EPI_RESID>(K);
    case 2: return occ_t<2, EPI_RESID>(K);
    case 4: return occ_t<4, EPI_RESID>(K);
    default: return occ_t<8, EPI_RESID>(K);
    }
}

cudaError_t launch_pdl(const void *fn, dim3 grid, dim3 block, void **args, cudaStream_t s) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelExC(&cfg, fn, args);
}

// --------------------------------------------------------------------------
// Task 20: final RMSNorm of 1..8 rows (stream_rmsnorm compute_stream.cpp:227-288)
// --------------------------------------------------------------------------
__global__ void __launch_bounds__(256) k_rmsnorm(const NormArgs a) {
    __shared__ int64_t red[8];
    __shared__ int32_t inv_s;
    pdl_wait();
    pdl_trigger();
    const int r = blockIdx.x;
    if (r >= a.step->rows) return;
    const int16_t *x = a.x + (size_t)r * a.n;
    if (a.inv_elems == 0) {
        if (threadIdx.x == 0) inv_s = a.inv_rms_const;
    } else {
        int64_t part = 0;
        for (int i = threadIdx.x; i < a.n; i += blockDim.x) part += (int64_t)x[i] * x[i];
        for (int o = 16; o >= 1; o >>= 1) part += shfl_xor64(part, o);
        if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = part;
        __syncthreads();
        if (threadIdx.x == 0) {
            int64_t s = 0;
            for (int w = 0; w < (int)(blockDim.x >> 5); w++) s += red[w];
            inv_s = inv_rms_q88(s > INT32_MAX ? INT32_MAX : (int32_t)s, a.inv_elems);
        }
    }
    __syncthreads();
    const int64_t inv = inv_s;
    for (int i = threadIdx.x; i < a.n; i += blockDim.x)
        a.y[(size_t)r * a.n + i] = (int16_t)sat16(rnd((int64_t)x[i] * inv * a.w[i], 16));
}

cudaError_t launch_rmsnorm(const NormArgs &a, int rows, cudaStream_t s) {
    NormArgs c = a;
    void *args[] = {&c};
    return launch_pdl((const void *)k_rmsnorm, dim3(rows), dim3(256), args, s);
}

// --------------------------------------------------------------------------
// tensor parallel: round the all-reduced exact sums and add the residual
// --------------------------------------------------------------------------
__global__ void k_round_resid(const ResidArgs a) {
    pdl_wait();
    pdl_trigger();
    const int rows = a.step->rows;
    const int total = rows * a.n;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x)
        a.out[i] = (int16_t)sat16((int32_t)a.resid[i] + round_mac(a.partial[i]));
}

cudaError_t launch_round_resid(const ResidArgs &a, int rows, cudaStream_t s) {
    ResidArgs c = a;
    void *args[] = {&c};
    const int blocks = (rows * a.n + 255) / 256;
    return launch_pdl((const void *)k_round_resid, dim3(blocks), dim3(256), args, s);
}

// --------------------------------------------------------------------------
// weight layout
// --------------------------------------------------------------------------
__global__ void k_pack_pairs(const int16_t *__restrict__ dense, int ld, int col0, int K,
                             const int32_t *__restrict__ row_of_slot, int nslots,
                             uint32_t *__restrict__ dst) {
    const int KW = K >> 1;
    const size_t total = (size_t)nslots * KW;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (size_t)gridDim.x * blockDim.x) {
        const int slot = (int)(i / KW);
        const int j = (int)(i - (size_t)slot * KW);
        const int16_t *row = dense + (size_t)row_of_slot[slot] * ld + col0;
        const uint32_t w0 = (uint16_t)row[2 * j], w1 = (uint16_t)row[2 * j + 1];
        dst[i] = (w0 & 0xffu) | ((w1 & 0xffu) << 8) | ((w0 >> 8) << 16) | ((w1 >> 8) << 24);
    }
}

cudaError_t launch_pack_pairs(const int16_t *dense, int ld, int col0, int K,
                              const int32_t *row_of_slot, int nslots, uint32_t *dst,
                              cudaStream_t s) {
    const size_t total = (size_t)nslots * (K >> 1);
    int blocks = (int)((total + 255) / 256);
    if (blocks > 65535 * 8) blocks = 65535 * 8;
    k_pack_pairs<<<blocks, 256, 0, s>>>(dense, ld, col0, K, row_of_slot, nslots, dst);
    return cudaGetLastError();
}

}  // namespace llmx
