// Projection kernel for blocks of 3..8 rows on the fifth-generation tensor
// cores (tcgen05.mma kind::i8, accumulators in tensor memory).
//
// Reference arithmetic: the exact int16 x int16 sum of the 8x64 fused MAC
// engine, rounded twice (kernel/mm_stream_8x64_fused_mac.cpp:11-22,89-96,
// 138-205; kernel/compute_core_8x64_unified.cpp:10-39; golden_projection
// host/host_qwen_8x64.cpp:3105-3142).
//
// Exactness.  Split every weight into a signed high byte and an unsigned low
// byte, w = 256*wh + wl, and every activation into a signed high byte and a
// signed low byte, x = 256*xh + xs + 128 with xs = (x & 255) - 128.  Then
//   sum w*x = 65536*sum(wh*xh) + 256*(sum(wh*xs) + sum(wl*xh)) + sum(wl*xs)
//             + 128*sum(w)
// Because xh and xs are both signed, the B operand [xh rows | xs rows] is one
// s8 matrix of N = 16 rows, and each weight plane needs one MMA per K-step:
// wh x B (s8 x s8) and wl x B (u8 x s8).  The int32 accumulators cannot
// overflow for K <= 11008 (|wh*xh|, |wh*xs| <= 2^14, |wl*xh|, |wl*xs| <=
// 255*128; 32640 * 11008 < 2^31).  sum(w) over the chunks a CTA accumulated
// comes from a per-tile-row prefix table of weight sums built at upload
// (k_mma_wsum).  The epilogue recombines in int64, so the result is the exact
// int64 dot product, as in the golden model -- the operand widths of the
// reference fit the tensor cores exactly once split into bytes.
//
// B200 mapping.  Weights are re-laid out at upload into "items": one item is
// one tile of 128 output rows x 128 inputs, as two 16 KiB byte planes (high,
// low) already in the tensor cores' K-major core-matrix order (8 rows x 16
// bytes per 128-byte core matrix), so one 1-D bulk copy moves an item from HBM
// into a shared-memory ring stage.  A projection is T tiles x C chunks of K;
// the T*C items are split evenly and contiguously over the CTAs (stream-K), so
// every CTA streams one contiguous byte range.  Per item the MMA thread issues
// 4 K-steps x 2 weight-plane products (M = 128, N = 16 = 8 activation rows x 2
// byte planes, K = 32 bytes) into one of two 32-column TMEM accumulator sets; four epilogue warps
// read the sums with tcgen05.ld (one TMEM lane = one output row) and run the
// fused epilogue of the path (RoPE + KV append, SiLU x up, residual, or the
// tensor-parallel partial sums).  A tile shared by two or more CTAs is
// finished by the last one to arrive: the others leave exact int64 partial
// sums in a scratch slot and count themselves in; nobody waits for anybody.
#include <cuda_runtime.h>

#include "device_util.cuh"
#include "fixed.cuh"
#include "kernels.cuh"
#include "gemv_common.cuh"

namespace llmx {

constexpr int kMmaThreads = 6 * 32;  // warp 0: TMEM + MMA issue, warp 1: weight producer, warps 2-5: epilogue
constexpr int kTmemCols = 64;        // two accumulator sets x {wh x [xh|xs], wl x [xh|xs]} x 8 rows
constexpr int kMmaHdr = 1024;        // barriers and flags at the start of dynamic shared memory
constexpr int kMmaMaxStages = 8;

// ---- tcgen05 primitives -----------------------------------------------------
// Shared-memory matrix descriptor, K-major, no swizzle: start address, LBO =
// byte distance between the two 16-byte core matrices along K of one MMA
// K-step, SBO = byte distance between 8-row core-matrix groups; version 1.
static __device__ __forceinline__ uint64_t umma_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    return (uint64_t)((saddr & 0x3FFFFu) >> 4) | ((uint64_t)(lbo >> 4) << 16) | ((uint64_t)(sbo >> 4) << 32) |
           (1ull << 46);
}
// Instruction descriptor, kind::i8: int32 accumulator, A and B K-major,
// M = 128, N = 16; a_signed / b_signed select s8 (1) or u8 (0).
static __host__ __device__ constexpr uint32_t umma_idesc_i8(int a_signed, int b_signed) {
    return (2u << 4) | ((uint32_t)a_signed << 7) | ((uint32_t)b_signed << 10) | ((16u >> 3) << 17) |
           ((128u >> 4) << 24);
}
static __device__ __forceinline__ void umma_i8(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n}" ::"r"(d_tmem),
        "l"(a), "l"(b), "r"(idesc), "r"(acc)
        : "memory");
}
// Arrive on an mbarrier once every tcgen05 operation this thread issued so far has completed.
static __device__ __forceinline__ void umma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
static __device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
static __device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
// 32 consecutive TMEM columns of this warp's 32 lanes (lane quarter in taddr bits 16+).
static __device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n"
        "tcgen05.wait::ld.sync.aligned;"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]),
          "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]),
          "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
        : "r"(taddr)
        : "memory");
}
static __device__ __forceinline__ void named_sync(int id, int threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// Item range of CTA b: [first_item(b), first_item(b + 1)).
static __host__ __device__ __forceinline__ int first_item(int b, int items, int grid) {
    return (int)((int64_t)items * b / grid);
}
// CTA whose range holds item i.
static __device__ __forceinline__ int cta_of_item(int i, int items, int grid) {
    int b = (int)(((int64_t)i * grid) / items);
    while (b + 1 < grid && first_item(b + 1, items, grid) <= i) b++;
    while (b > 0 && first_item(b, items, grid) > i) b--;
    return b;
}

// RMSNorm factors of the activation rows (inv_s), when a norm row is given.
static __device__ void mma_norm_rows(const MmaArgs &a, int rows, int tid, int T, int32_t *inv_s, int64_t *red) {
    const int K = a.K;
    if (a.norm != nullptr) {
        if (a.inv_elems == 0) {
            if (tid < kMaxRows) inv_s[tid] = a.inv_rms_const;
        } else {  // general RMSNorm: full-row sums of squares (stream_rmsnorm compute_stream.cpp:242-283)
            // T / 8 threads per row, 16-byte loads, four in flight per thread: every
            // row's sum in one pass (the rows are independent)
            if (tid < kMaxRows) red[tid] = 0;
            named_sync(2, T);
            const int tpr = T / kMaxRows, r = tid / tpr, sub = tid - r * tpr;
            if (r < rows) {
                const uint4 *x4 = reinterpret_cast<const uint4 *>(a.x + (size_t)r * K);
                const int KV8 = K >> 3;
                int64_t part = 0;
                for (int v0 = sub; v0 < KV8; v0 += 4 * tpr) {
                    uint4 q[4];
#pragma unroll
                    for (int k = 0; k < 4; k++) {
                        const int v = v0 + k * tpr;
                        q[k] = v < KV8 ? x4[v] : make_uint4(0, 0, 0, 0);
                    }
#pragma unroll
                    for (int k = 0; k < 4; k++) {
                        const uint32_t w[4] = {q[k].x, q[k].y, q[k].z, q[k].w};
#pragma unroll
                        for (int i = 0; i < 4; i++)
                            part += (int64_t)lo16(w[i]) * lo16(w[i]) + (int64_t)hi16(w[i]) * hi16(w[i]);
                    }
                }
                atomicAdd(reinterpret_cast<unsigned long long *>(red + r), (unsigned long long)part);
            }
            named_sync(2, T);
            if (tid < kMaxRows) {
                const int64_t sum = red[tid];
                inv_s[tid] = inv_rms_q88(sum > INT32_MAX ? INT32_MAX : (int32_t)sum, a.inv_elems);
            }
        }
        named_sync(2, T);
    }
}

// Activation rows -> the byte planes of every item chunk this CTA needs (slot j
// = chunk of item w0 + j), RMS-normalised when a norm row is given, in item
// order by the T threads of named barrier 4: after each round the count of
// finished slots is published in *staged (release), so the MMA thread starts on
// the first items while the later ones are still being staged.
// Slot layout (2 KiB): high plane then low plane, each 8 rows x 128 bytes in
// core-matrix order (16-byte column group kc at kc * 128, row r at r * 16).
static __device__ void mma_stage_rows(const MmaArgs &a, char *bsl, int w0, int n, int rows, int tid, int T,
                                      const int32_t *inv_s, int *staged) {
    const int K = a.K;
    // one 16-element group (row r, column group kc of the chunk) per unit; the
    // loads of kBatch units are all in flight before any is used
    constexpr int kBatch = 4;
    const int units = n * kMaxRows * 8;
    for (int base = 0; base < units; base += kBatch * T) {
        const int u0 = base + tid;
        uint4 xv[kBatch][2], wv[kBatch][2];
#pragma unroll
        for (int k = 0; k < kBatch; k++) {
            const int u = u0 + k * T;
            const int j = u / (kMaxRows * 8), rem = u - j * (kMaxRows * 8), r = rem >> 3, kc = rem & 7;
            const int col = ((w0 + j) % a.C) * 128 + kc * 16;
            // K is a multiple of 8: a 16-column group is whole, half or not present
#pragma unroll
            for (int h = 0; h < 2; h++) {
                const bool in = u < units && r < rows && col + 8 * h < K;
                xv[k][h] = in ? *reinterpret_cast<const uint4 *>(a.x + (size_t)r * K + col + 8 * h) : make_uint4(0, 0, 0, 0);
                wv[k][h] = in && a.norm != nullptr ? *reinterpret_cast<const uint4 *>(a.norm + col + 8 * h)
                                                   : make_uint4(0, 0, 0, 0);
            }
        }
#pragma unroll
        for (int k = 0; k < kBatch; k++) {
            const int u = u0 + k * T;
            if (u >= units) break;
            const int j = u / (kMaxRows * 8), rem = u - j * (kMaxRows * 8), r = rem >> 3, kc = rem & 7;
            const int32_t inv = a.norm != nullptr ? inv_s[r] : 0;
            uint32_t hw[4], lw[4];
#pragma unroll
            for (int h = 0; h < 2; h++) {
                uint32_t xw[4] = {xv[k][h].x, xv[k][h].y, xv[k][h].z, xv[k][h].w};
                const uint32_t ww[4] = {wv[k][h].x, wv[k][h].y, wv[k][h].z, wv[k][h].w};
                if (a.norm != nullptr) {
#pragma unroll
                    for (int q = 0; q < 4; q++) {  // x * w fits 32 bits; one widening multiply by inv
                        const int32_t y0 = sat16(rnd((int64_t)(lo16(xw[q]) * lo16(ww[q])) * inv, 16));
                        const int32_t y1 = sat16(rnd((int64_t)(hi16(xw[q]) * hi16(ww[q])) * inv, 16));
                        xw[q] = ((uint32_t)y0 & 0xffffu) | ((uint32_t)y1 << 16);
                    }
                }
                // bytes of 4 consecutive int16 (two words): high bytes 1,3,5,7 and low
                // bytes 0,2,4,6, the low bytes stored as signed (x & 255) - 128
                hw[2 * h] = __byte_perm(xw[0], xw[1], 0x7531);
                lw[2 * h] = __byte_perm(xw[0], xw[1], 0x6420) ^ 0x80808080u;
                hw[2 * h + 1] = __byte_perm(xw[2], xw[3], 0x7531);
                lw[2 * h + 1] = __byte_perm(xw[2], xw[3], 0x6420) ^ 0x80808080u;
            }
            char *slot = bsl + (size_t)j * 2048 + kc * 128 + r * 16;
            *reinterpret_cast<uint4 *>(slot) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
            *reinterpret_cast<uint4 *>(slot + 1024) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // visible to the tensor cores
        named_sync(4, T);
        if (tid == 0) {
            const int done = min(n, (base + kBatch * T) / (kMaxRows * 8));
            asm volatile("st.release.cta.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(staged)), "r"(done) : "memory");
        }
    }
}

static __device__ __forceinline__ int ld_acquire_smem(const int *p) {
    int v;
    asm volatile("ld.acquire.cta.shared::cta.b32 %0, [%1];" : "=r"(v) : "r"(smem_u32(p)) : "memory");
    return v;
}

// Final epilogue of one tile: thread m (TMEM lane) holds the exact sums of
// tile row m for the 8 activation rows.
template <int EPI>
static __device__ void mma_epilogue(const MmaArgs &a, const Step &st, int t, int m, const int64_t (&S)[kMaxRows],
                                    int32_t *ys, const int16_t *etab_s) {
    const int rows = st.rows;
    if constexpr (EPI == EPI_RESID || EPI == EPI_PARTIAL) {
        const int o = t * 128 + m;
        if (o >= a.n_out) return;
        if constexpr (EPI == EPI_RESID) {
#pragma unroll
            for (int r = 0; r < kMaxRows; r++)
                if (r < rows) {
                    const size_t i = (size_t)r * a.out_stride + o;
                    a.out[i] = (int16_t)sat16((int32_t)a.resid[i] + round_mac(S[r]));
                }
        } else if (a.ar.n > 1) {  // tensor parallel: straight into every rank's exchange region
            const uint32_t n = st.ar_base + a.ar_off;
#pragma unroll
            for (int r = 0; r < kMaxRows; r++)
                if (r < rows) {
                    const size_t w = ar_word_index((int)(n & 1u), a.ar.me, r, a.ar.hidden, o);
                    const uint64_t word = ar_pack(S[r], ar_tag(n));
                    for (int p = 0; p < a.ar.n; p++)
                        ar_store(reinterpret_cast<uint64_t *>(a.ar.base[p] + kArHeader) + w, word);
                }
        } else {
#pragma unroll
            for (int r = 0; r < kMaxRows; r++)
                if (r < rows) a.partial[(size_t)r * a.out_stride + o] = S[r];
        }
    } else {
    // pair epilogues: rows m and m + 64 of the tile form one unit; thread m
    // then finishes pair (m mod 64) for activation rows 4*(m / 64) .. +3
#pragma unroll
    for (int r = 0; r < kMaxRows; r++) ys[r * 128 + m] = round_mac(S[r]);
    named_sync(3, 128);
    const int p = m & 63, r0 = (m >> 6) * 4;
    if constexpr (EPI == EPI_SILU) {
        const int u = t * 64 + p;  // FFN column of this rank
        if (u < a.n_out) {
#pragma unroll
            for (int k = 0; k < 4; k++) {
                const int r = r0 + k;
                if (r < rows)
                    a.out[(size_t)r * a.out_stride + u] = (int16_t)silu_mul(ys[r * 128 + p], ys[r * 128 + p + 64], etab_s);
            }
        }
    } else {  // EPI_QKV: tile = one head (q heads of this rank, then K heads, then V heads)
        constexpr int half = 64;
        const bool rope = t < a.q_tiles + a.kv_tiles;
        int64_t cs[4], sn[4];
#pragma unroll
        for (int k = 0; k < 4; k++) {  // RoPE rows of every position first (independent loads)
            const int pos = st.position + r0 + k;
            cs[k] = rope && r0 + k < rows ? a.rope[(size_t)pos * 128 + p] : 0;
            sn[k] = rope && r0 + k < rows ? a.rope[(size_t)pos * 128 + half + p] : 0;
        }
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const int r = r0 + k;
            if (r >= rows) continue;
            const int pos = st.position + r;
            const int32_t y0 = ys[r * 128 + p], y1 = ys[r * 128 + p + half];
            if (rope) {
                // RoPE rotate_fix16_pair_with_quantized_rope host:4765-4788
                const int16_t z0 = (int16_t)sat16(rnd((int64_t)y0 * cs[k] - (int64_t)y1 * sn[k], 8));
                const int16_t z1 = (int16_t)sat16(rnd((int64_t)y1 * cs[k] + (int64_t)y0 * sn[k], 8));
                int16_t *dst = t < a.q_tiles ? a.out + (size_t)r * a.out_stride + (size_t)t * 128
                                             : a.kc + ((size_t)(t - a.q_tiles) * a.max_seq + pos) * 128;
                dst[p] = z0;
                dst[p + half] = z1;
            } else {
                int16_t *dst = a.vc + ((size_t)(t - a.q_tiles - a.kv_tiles) * a.max_seq + pos) * 128;
                dst[p] = (int16_t)y0;
                dst[p + half] = (int16_t)y1;
            }
        }
    }
    named_sync(3, 128);  // ys free for the next tile
    }
}

template <int EPI>
__global__ void __launch_bounds__(kMmaThreads, 1) k_mma_proj(const MmaArgs a) {
    LLMX_TL_GUARD(a.tl_slot);
    extern __shared__ __align__(1024) char smem[];
    // header: barriers, flags and the staging reduction (kMmaHdr bytes)
    uint64_t *full = reinterpret_cast<uint64_t *>(smem);  // [kMmaMaxStages]
    uint64_t *empty = full + kMmaMaxStages;               // [kMmaMaxStages]
    uint64_t *tfull = empty + kMmaMaxStages;              // [2] accumulator set b ready for the epilogue
    uint64_t *tempty = tfull + 2;                         // [2] accumulator set b read out
    uint64_t *done = tempty + 2;                          // every MMA of the CTA completed
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(done + 1);
    int *last_s = reinterpret_cast<int *>(tmem_slot + 1);
    int *fail_s = last_s + 1;                              // [2][4] per-tile wait outcome of each epilogue warp
    int32_t *inv_s = fail_s + 8;                           // [8]
    int *staged_s = reinterpret_cast<int *>(inv_s + 8);    // activation slots staged so far
    int64_t *red = reinterpret_cast<int64_t *>(smem + 512);  // [8][8]
    char *ring = smem + kMmaHdr;
    const int S = a.stages;
    char *bsl = ring + (size_t)S * kMmaItemBytes;
    int32_t *ys = reinterpret_cast<int32_t *>(bsl + (size_t)a.max_items * 2048);  // [8][128]
    int16_t *etab_s = reinterpret_cast<int16_t *>(ys + kMaxRows * 128);            // [2049] SiLU exp table
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int items = a.T * a.C;
    const int w0 = first_item(blockIdx.x, items, gridDim.x), w1 = first_item(blockIdx.x + 1, items, gridDim.x);
    const int n = w1 - w0;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; s++) {
            mbar_init(full + s, 1);
            mbar_init(empty + s, 1);  // one tcgen05.commit per consumed item
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(tfull + b, 1);
            mbar_init(tempty + b, 128);  // every epilogue thread
        }
        mbar_init(done, 1);
        *staged_s = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 1) {  // ---------------- weight producer --------------------------------
        if (lane == 0) {
            const uint64_t policy = evict_first_policy();
            const char *src = reinterpret_cast<const char *>(a.w) + (size_t)w0 * kMmaItemBytes;
            bool ok = true;
            int issued = 0;
            for (int j = 0; j < n; j++) {
                const int s = j % S;
                if (j >= S && !mbar_wait(empty + s, ((j / S) - 1) & 1)) {
                    ok = false;
                    break;
                }
                mbar_expect_tx(full + s, kMmaItemBytes);
                bulk_g2s_hint(ring + (size_t)s * kMmaItemBytes, src + (size_t)j * kMmaItemBytes, kMmaItemBytes,
                              full + s, policy);
                issued = j + 1;
                if (j == S - 1) pdl_wait();  // ring primed before waiting on the previous kernel
            }
            if (n < S) pdl_wait();
            if (!ok) {
                atomicExch(a.error, 1);
                for (int s = 0; s < S && s < issued; s++) {
                    const int last = s + ((issued - 1 - s) / S) * S;
                    (void)mbar_wait(full + s, (last / S) & 1);
                }
            }
        }
    } else {  // ---------------- warps 0, 2-5: activations, then MMA / epilogue ---------
        const int tid = warp == 0 ? lane : threadIdx.x - 32;  // 0..159
        const Step st = load_step(a.step);
        if (EPI == EPI_SILU)  // the SiLU table does not depend on the previous kernel either
            for (int i = tid; i < 2049; i += 160) etab_s[i] = a.etab[i];
        pdl_wait();
        pdl_trigger();
        mma_norm_rows(a, st.rows, tid, 160, inv_s, red);

        if (warp == 0) {  // ---------------- MMA issue (one thread) ----------------------
            if (lane == 0) {
                constexpr uint32_t kSS = umma_idesc_i8(1, 1), kUS = umma_idesc_i8(0, 1);
                int tiles_done = 0;
                bool ok = true;
                for (int j = 0; j < n && ok; j++) {
                    const int i = w0 + j, c = i % a.C;
                    const bool first = j == 0 || c == 0, last = j == n - 1 || c == a.C - 1;
                    const int b = tiles_done & 1;
                    if (first && tiles_done >= 2 && !mbar_wait(tempty + b, ((tiles_done >> 1) - 1) & 1)) ok = false;
                    if (ok && !mbar_wait(full + j % S, (j / S) & 1)) ok = false;
                    if (ok && ld_acquire_smem(staged_s) <= j) {  // this item's activation slot (bounded wait)
                        ok = false;
                        for (uint32_t it = 0; it < kSpinLimit; it++)
                            if (ld_acquire_smem(staged_s) > j) {
                                ok = true;
                                break;
                            }
                    }
                    if (!ok) break;
                    tc_fence_after();
                    const uint32_t ah = smem_u32(ring + (size_t)(j % S) * kMmaItemBytes), al = ah + 16384;
                    // B: the slot's high plane (rows 0-7) and signed low plane (rows 8-15),
                    // one 8-row core-matrix group apart (SBO 1024): one N = 16 operand
                    const uint32_t bh = smem_u32(bsl + (size_t)j * 2048);
                    const uint32_t d = tmem + (uint32_t)b * 32;
#pragma unroll
                    for (int k = 0; k < 4; k++) {  // 32-byte K-steps of the 128-byte chunk
                        const uint32_t acc = (first && k == 0) ? 0u : 1u;
                        const uint64_t dah = umma_desc(ah + k * 256, 128, 1024), dal = umma_desc(al + k * 256, 128, 1024);
                        const uint64_t db = umma_desc(bh + k * 256, 128, 1024);
                        umma_i8(d + 0, dah, db, kSS, acc);   // columns 0-7 wh.xh, 8-15 wh.xs
                        umma_i8(d + 16, dal, db, kUS, acc);  // columns 16-23 wl.xh, 24-31 wl.xs
                    }
                    umma_commit(empty + j % S);  // ring stage free once these MMAs are done
                    if (last) {
                        umma_commit(tfull + b);
                        tiles_done++;
                    }
                }
                if (!ok) atomicExch(a.error, 2);  // the epilogue finds the flag and stops waiting
                // the accumulators are released only after every issued MMA has completed
                umma_commit(done);
                if (!mbar_wait(done, 0)) atomicExch(a.error, 2);
            }
            __syncwarp();
        } else {  // ---------------- epilogue warps 2-5: activation slots, then the tiles -------
            mma_stage_rows(a, bsl, w0, n, st.rows, (int)threadIdx.x - 64, 128, inv_s, staged_s);
            const int q = warp & 3, m = q * 32 + lane;  // TMEM lane quarter of this warp, tile row
            const int t0 = w0 / a.C, t1 = n > 0 ? (w1 - 1) / a.C : t0 - 1;
            int tiles_done = 0;
            for (int t = t0; t <= t1; t++, tiles_done++) {
                const int b = tiles_done & 1;
                // the four warps decide together whether to go on (they meet at named barriers)
                const bool okw = mbar_wait_err(tfull + b, (tiles_done >> 1) & 1, a.error);
                if (lane == 0) fail_s[b * 4 + q] = okw ? 0 : 1;
                named_sync(3, 128);
                if (fail_s[b * 4] | fail_s[b * 4 + 1] | fail_s[b * 4 + 2] | fail_s[b * 4 + 3]) {
                    if (m == 0) atomicCAS(a.error, 0, 3);
                    break;
                }
                tc_fence_after();
                uint32_t v[32];
                tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)b * 32, v);
                tc_fence_before();
                mbar_arrive(tempty + b);
                const int seg0 = max(w0, t * a.C), seg1 = min(w1, (t + 1) * a.C);
                // + 128 * (sum of this tile row's weights over the chunks accumulated here)
                const int32_t *ws = a.wsum + (size_t)t * (a.C + 1) * 128 + m;
                const int64_t corr =
                    128 * (int64_t)(ws[(size_t)(seg1 - t * a.C) * 128] - ws[(size_t)(seg0 - t * a.C) * 128]);
                int64_t Sm[kMaxRows];
#pragma unroll
                for (int r = 0; r < kMaxRows; r++)
                    Sm[r] = (int64_t)(int32_t)v[r] * 65536 +
                            ((int64_t)(int32_t)v[8 + r] + (int64_t)(int32_t)v[16 + r]) * 256 + (int64_t)(int32_t)v[24 + r] +
                            corr;
                if (seg0 != t * a.C || seg1 != (t + 1) * a.C) {
                    // shared tile: leave the partial sums, count in; the last CTA finishes it
                    const int which = t == t0 ? 0 : 1;
                    int64_t *slot = a.scratch + ((size_t)(blockIdx.x * 2 + which) * kMaxRows) * 128;
#pragma unroll
                    for (int r = 0; r < kMaxRows; r++) slot[r * 128 + m] = Sm[r];
                    named_sync(3, 128);  // every thread's slot writes happen before thread 0's release below
                    const int b_lo = cta_of_item(t * a.C, items, gridDim.x);
                    const int b_hi = cta_of_item((t + 1) * a.C - 1, items, gridDim.x);
                    if (m == 0) {
                        int old;
                        asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], 1;" : "=r"(old) : "l"(a.tile_cnt + t) : "memory");
                        *last_s = old == b_hi - b_lo;
                    }
                    named_sync(3, 128);
                    if (!*last_s) continue;
                    for (int b0 = b_lo; b0 <= b_hi; b0 += 4) {  // 4 contributors' loads in flight
                        int64_t part[4][kMaxRows];
#pragma unroll
                        for (int k = 0; k < 4; k++) {
                            const int bb = b0 + k;
                            const bool use = bb <= b_hi && bb != (int)blockIdx.x;
                            const int wh = use && t != first_item(bb, items, gridDim.x) / a.C ? 1 : 0;
                            const int64_t *o = a.scratch + ((size_t)((use ? bb : 0) * 2 + wh) * kMaxRows) * 128;
#pragma unroll
                            for (int r = 0; r < kMaxRows; r++) part[k][r] = use ? __ldcg(o + r * 128 + m) : 0;
                        }
#pragma unroll
                        for (int k = 0; k < 4; k++)
#pragma unroll
                            for (int r = 0; r < kMaxRows; r++) Sm[r] += part[k][r];
                    }
                    if (m == 0) a.tile_cnt[t] = 0;  // ready for the next launch
                }
                mma_epilogue<EPI>(a, st, t, m, Sm, ys, etab_s);
            }
        }
    }
    // every MMA has completed before the accumulators are released: the epilogue
    // waited for each tile's commit, and an error path waits for the last one here
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
    }
}

size_t mma_smem_bytes(int stages, int max_items) {
    return kMmaHdr + (size_t)stages * kMmaItemBytes + (size_t)max_items * 2048 + (size_t)kMaxRows * 128 * 4 + 4224;
}

// Ring depth that fits shared memory (2..kMaxStages stages).
int mma_stages(int max_items, int max_smem) {
    int s = 6 < kMmaMaxStages ? 6 : kMmaMaxStages;
    while (s > 2 && mma_smem_bytes(s, max_items) > (size_t)max_smem) s--;
    return mma_smem_bytes(s, max_items) <= (size_t)max_smem ? s : 0;
}

template <int EPI>
static cudaError_t launch_mma_t(const MmaArgs &a, int grid, cudaStream_t st) {
    MmaArgs c = a;
    LLMX_TL_TAKE(c, EPI == EPI_QKV ? "mma/qkv" : EPI == EPI_RESID ? "mma/resid" : EPI == EPI_SILU ? "mma/gate_up" : "mma/partial");
    void *args[] = {&c};
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kMmaThreads);
    cfg.dynamicSmemBytes = mma_smem_bytes(a.stages, a.max_items);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelExC(&cfg, (const void *)k_mma_proj<EPI>, args);
}

cudaError_t launch_mma_proj(const MmaArgs &a, int epi, int grid, cudaStream_t s) {
    switch (epi) {
    case EPI_QKV: return launch_mma_t<EPI_QKV>(a, grid, s);
    case EPI_RESID: return launch_mma_t<EPI_RESID>(a, grid, s);
    case EPI_SILU: return launch_mma_t<EPI_SILU>(a, grid, s);
    default: return launch_mma_t<EPI_PARTIAL>(a, grid, s);
    }
}

cudaError_t mma_configure(int max_smem_bytes) {
    constexpr auto kAttr = cudaFuncAttributeMaxDynamicSharedMemorySize;
    cudaError_t e;
    if ((e = cudaFuncSetAttribute(k_mma_proj<EPI_QKV>, kAttr, max_smem_bytes))) return e;
    if ((e = cudaFuncSetAttribute(k_mma_proj<EPI_RESID>, kAttr, max_smem_bytes))) return e;
    if ((e = cudaFuncSetAttribute(k_mma_proj<EPI_SILU>, kAttr, max_smem_bytes))) return e;
    return cudaFuncSetAttribute(k_mma_proj<EPI_PARTIAL>, kAttr, max_smem_bytes);
}

// --------------------------------------------------------------------------
// weight layout for the tensor-core path (model upload)
// --------------------------------------------------------------------------
// Item (t, c) = tile t (128 output rows; tile row m is dense row rows_of[t*128+m],
// -1 = zero padding), K-chunk c (input columns col0 + c*128 .. +127, zero past K):
// high-byte plane then low-byte plane, each with byte (m, k) at
// ((m / 8) * 8 + k / 16) * 128 + (m % 8) * 16 + k % 16.
__global__ void k_pack_mma(const int16_t *__restrict__ dense, int ld, int col0, int K, int C,
                           const int32_t *__restrict__ rows_of, int T, uint8_t *__restrict__ dst) {
    const size_t groups = (size_t)T * C * 2 * 128 * 8;  // 16-byte groups
    for (size_t g = (size_t)blockIdx.x * blockDim.x + threadIdx.x; g < groups; g += (size_t)gridDim.x * blockDim.x) {
        const int kc = (int)(g & 7), m = (int)((g >> 3) & 127);
        const size_t rest = g >> 10;
        const int plane = (int)(rest & 1);
        const size_t item = rest >> 1;
        const int t = (int)(item / C), c = (int)(item - (size_t)t * C);
        const int row = rows_of[t * 128 + m];
        uint32_t w[4] = {0, 0, 0, 0};
        for (int e = 0; e < 16; e++) {
            const int col = c * 128 + kc * 16 + e;
            uint32_t byte = 0;
            if (row >= 0 && col < K) {
                const uint32_t v = (uint16_t)dense[(size_t)row * ld + col0 + col];
                byte = plane == 0 ? (v >> 8) : (v & 0xffu);
            }
            w[e >> 2] |= byte << (8 * (e & 3));
        }
        uint8_t *p = dst + item * kMmaItemBytes + (size_t)plane * 16384 + ((m >> 3) * 8 + kc) * 128 + (m & 7) * 16;
        *reinterpret_cast<uint4 *>(p) = make_uint4(w[0], w[1], w[2], w[3]);
    }
}

cudaError_t launch_pack_mma(const int16_t *dense, int ld, int col0, int K, int C, const int32_t *rows_of, int T,
                            uint8_t *dst, cudaStream_t s) {
    const size_t groups = (size_t)T * C * 2 * 128 * 8;
    int blocks = (int)std::min<size_t>((groups + 255) / 256, 65535 * 8);
    k_pack_mma<<<blocks, 256, 0, s>>>(dense, ld, col0, K, C, rows_of, T, dst);
    return cudaGetLastError();
}

// Prefix over K-chunks of every tile row's weight sums: wsum[(t*(C+1) + c)*128 + m]
// = sum of the row's weights in chunks [0, c) (|value| < 2^29 for K <= 11008).
__global__ void k_mma_wsum(const int16_t *__restrict__ dense, int ld, int col0, int K, int C,
                           const int32_t *__restrict__ rows_of, int T, int32_t *__restrict__ wsum) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;  // tile row t*128 + m
    if (i >= T * 128) return;
    const int t = i >> 7, m = i & 127, row = rows_of[i];
    int32_t acc = 0;
    wsum[(size_t)t * (C + 1) * 128 + m] = 0;
    for (int c = 0; c < C; c++) {
        if (row >= 0)
            for (int k = c * 128; k < min(K, (c + 1) * 128); k++) acc += dense[(size_t)row * ld + col0 + k];
        wsum[((size_t)t * (C + 1) + c + 1) * 128 + m] = acc;
    }
}

cudaError_t launch_mma_wsum(const int16_t *dense, int ld, int col0, int K, int C, const int32_t *rows_of, int T,
                            int32_t *wsum, cudaStream_t s) {
    k_mma_wsum<<<(T * 128 + 127) / 128, 128, 0, s>>>(dense, ld, col0, K, C, rows_of, T, wsum);
    return cudaGetLastError();
}

}  // namespace llmx

LLMX_TL_READER(mma_proj)
