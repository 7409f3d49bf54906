// Tile-exact online-softmax attention of the resident layer path.
//
// Reference: run_cc8_resident_decode_attention kernel/control_cache_8x64.cpp:5492-5765
// and its golden model golden_tiled_flash_attention_q2_14_impl<true>
// host/host_qwen_8x64.cpp:3610-3739 (QK scores of golden_attention_mm :3219-3278).
//
// The reference walks the context in 64-position tiles in order, carrying a
// running max m, a Q16.16 normaliser sum and a Q16.16 accumulator that are
// rescaled by P(m_old - m_new) at every tile.  Those recurrences round at
// every step, so the tile order must be replayed exactly -- but only the cheap
// (sum, acc) update is sequential: the running max after tile t is the prefix
// max of tile maxima, and a tile's probabilities / PV only need that value.
//
// One thread-block cluster of C CTAs (8, or 16 when few heads leave SMs idle)
// handles one (row, query head).
// CTA c owns the contiguous tiles [c*tpc, (c+1)*tpc):
//   1. K rows of its tiles land in shared memory (cp.async); QK scores of its
//      positions; the buffer is refilled with the V rows while each owned
//      tile's maximum is stored into every CTA's shared memory (DSMEM push);
//   2. cluster barrier; running maxima (prefix max of the pushed maxima),
//      Q2.14 probabilities, tile sums and rescale factors (pushed to every
//      CTA) and the raw-payload PV tile values, each pushed to the CTA that
//      finalises that output element;
//   3. cluster barrier; the (sum, acc) recurrence in tile order on local
//      shared memory, each CTA finalising hd/C output elements.
// All remote accesses are stores issued before a barrier, so after each
// barrier a CTA reads only its own shared memory, and no CTA needs to wait for
// the others before it exits.  All waits are hardware cluster barriers: no
// flags, no spin loops, and no global scratch memory.
#include <cooperative_groups.h>
#include <cuda_runtime.h>

#include "device_util.cuh"
#include "fixed.cuh"
#include "kernels.cuh"
#include "gemv_common.cuh"

namespace llmx {

namespace cg = cooperative_groups;

constexpr int kAttnThreads = 256;
constexpr int kMaxHd = 128;

static __device__ __forceinline__ void cp_async16(void *dst, const void *src) {
    const unsigned d = (unsigned)__cvta_generic_to_shared(dst);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(d), "l"(src) : "memory");
}
static __device__ __forceinline__ void cp_async_wait_all() {
    asm volatile("cp.async.commit_group;\ncp.async.wait_group 0;" ::: "memory");
}

constexpr int kMaxTiles = kCluster * kMaxTilesPerCta;
// the softmax exp table (2049 entries, padded to 2056 in device memory) moves
// as 257 16-byte cp.async chunks
constexpr int kPtabChunks = 257;
constexpr int kErrAttnCopy = 3;  // device error code: a K/V copy did not complete in time

// K rows and V rows of a CTA's positions arrive with one 1-D bulk copy each
// (completion on an mbarrier): the rows are contiguous in the cache and stay
// unpadded in shared memory (head_dim int16 per row).  Lane L of the QK loop
// walks the 16-byte vectors of its row starting at vector L mod (head_dim/8),
// so the eight lanes of a quarter warp read eight different bank groups.
static __device__ __forceinline__ int rot_vec(int v, int vpr) { return v >= vpr ? v - vpr : v; }

struct AttnSmem {      // carved out of dynamic shared memory
    int16_t *kv;       // [tpc*64][hd] raw Q8.8 K rows, then V rows, of the owned tiles
    int16_t *ptab;     // [2049] softmax exp table
    int16_t *q;        // [hd]
    int16_t *sc;       // [tpc*64] scores, then Q2.14 probabilities
    int16_t *tvr;      // [kMaxTiles][hd/C] tile values of the elements this CTA finalises
    int32_t *mloc;     // [kMaxTiles] every tile's maximum (pushed by the owners)
    int32_t *gsum;     // [kMaxTiles] every tile's sum (pushed)
    int32_t *gold;     // [kMaxTiles] every tile's rescale factor (pushed)
    int32_t *tsum;     // [tpc] owned tile sums (local accumulation)
    uint64_t *bar;     // [3] completion of the K, the V and the O-weight copies
    int16_t *att;      // [hd] the head's output (fused O projection)
    uint32_t *ow;      // [o_rows][hd/2] this CTA's O rows, the head's columns (fused O projection):
                       // the K/V buffer, reused once PV is done
};

static __host__ __device__ size_t align16(size_t b) { return (b + 15) & ~size_t(15); }

// split = false: the O slice reuses the K/V buffer once PV is done (the same
// bytes: the CTA count per SM stays that of attention alone, which keeps every
// cluster of the grid resident at once), and each CTA holds the tile values of
// the hd/cl output elements it finalises.  split = true (the k_attn<C, true>
// variant): the O slice has a buffer of its own, filled from the kernel's start,
// and every CTA holds the tile values of all hd elements.
static __host__ __device__ size_t attn_layout(int tpc, int hd, int cl, int o_rows, size_t off[12],
                                              bool split = false) {
    const size_t rows = (size_t)tpc * kTile;
    size_t b = 0;
    const size_t kv_rows = split || rows > (size_t)o_rows ? rows : (size_t)o_rows;
    off[0] = b; b = align16(b + kv_rows * kMaxHd * 2);                       // kv (+ O slice)
    off[1] = b; b = align16(b + kPtabChunks * 16);                           // ptab
    off[2] = b; b = align16(b + (size_t)kMaxHd * 2);                         // q
    off[3] = b; b = align16(b + rows * 2);                                   // sc
    off[4] = b; b = align16(b + (size_t)kMaxTiles * (split ? kMaxHd : kMaxHd / cl) * 2);  // tvr
    off[5] = b; b = align16(b + (size_t)kMaxTiles * 4);                      // mloc
    off[6] = b; b = align16(b + (size_t)kMaxTiles * 4);                      // gsum
    off[7] = b; b = align16(b + (size_t)kMaxTiles * 4);                      // gold
    off[8] = b; b = align16(b + (size_t)tpc * 4);                            // tsum
    off[9] = b; b = align16(b + 3 * 8);                                      // bar
    off[10] = b; b = align16(b + (size_t)kMaxHd * 2);                        // att
    if (split) {
        off[11] = b; b = align16(b + (size_t)o_rows * kMaxHd * 2);           // ow
    } else {
        off[11] = off[0];                                                    // ow
    }
    (void)hd;
    return b;
}

size_t attn_smem_bytes(int tpc, int hd, int cluster, int o_rows, bool split) {
    size_t off[12];
    return attn_layout(tpc, hd, cluster, o_rows, off, split);
}


// kSplit (O projection fused only, LLMX_ATTN_SPLIT_O): the O slice is copied
// into a buffer of its own from the kernel's start, and the PV tile values go
// to every CTA, which then runs the recurrence of all hd elements itself -- no
// third cluster barrier (the head-output exchange) before the O rows.
// kTp (O projection fused on a tensor-parallel rank, LLMX_ATTN_FUSE_O_TP): the
// rank's O sums of a slice of O rows are complete once the CTA of that slice of
// every local head has added its part; the last of them to arrive pushes the
// slice to every rank's exchange region (the words the O projection's
// EPI_PARTIAL epilogue would store) and clears the sums and the count.
template <int C, bool kSplit, bool kTp>
__global__ void __launch_bounds__(kAttnThreads) k_attn(const AttnArgs a) {
    LLMX_TL_GUARD(a.tl_slot);
    extern __shared__ __align__(16) char raw[];
    cg::cluster_group cluster = cg::this_cluster();
    const int c = (int)cluster.block_rank();
    const int lh = blockIdx.x / C;  // local query head
    const int r = blockIdx.y;
    const int hd = a.hd, vpr = hd >> 3, epc = hd / C;  // elements finalised per CTA
    size_t off[12];
    attn_layout(a.tpc_max, hd, C, a.o_w != nullptr ? a.o_rows : 0, off, kSplit);
    AttnSmem m;
    m.kv = reinterpret_cast<int16_t *>(raw + off[0]);
    m.ptab = reinterpret_cast<int16_t *>(raw + off[1]);
    m.q = reinterpret_cast<int16_t *>(raw + off[2]);
    m.sc = reinterpret_cast<int16_t *>(raw + off[3]);
    m.tvr = reinterpret_cast<int16_t *>(raw + off[4]);
    m.mloc = reinterpret_cast<int32_t *>(raw + off[5]);
    m.gsum = reinterpret_cast<int32_t *>(raw + off[6]);
    m.gold = reinterpret_cast<int32_t *>(raw + off[7]);
    m.tsum = reinterpret_cast<int32_t *>(raw + off[8]);
    m.bar = reinterpret_cast<uint64_t *>(raw + off[9]);
    m.att = reinterpret_cast<int16_t *>(raw + off[10]);
    m.ow = reinterpret_cast<uint32_t *>(raw + off[11]);

    // the exp table, the step record and the O weights do not depend on the producer kernel
    for (int i = threadIdx.x; i < kPtabChunks; i += blockDim.x) cp_async16(m.ptab + 8 * i, a.ptab + 8 * i);
    const Step st = load_step(a.step);
    const bool row_ok = r < st.rows;
    // fused O projection: this CTA's o_rows O rows of the head's hd columns
    // (contiguous in the head-major copy) are warmed into L2 now -- they do not
    // depend on the producer kernel -- and copied into the K/V buffer once PV is done
    const bool fuse_o = a.o_w != nullptr && row_ok;
    const uint32_t ow_bytes = (uint32_t)a.o_rows * hd * 2;
    const uint32_t *ow_src = a.o_w + ((size_t)lh * a.hidden + (size_t)c * a.o_rows) * (hd >> 1);
    if (threadIdx.x == 0) {
        mbar_init(m.bar, 1);
        mbar_init(m.bar + 1, 1);
        mbar_init(m.bar + 2, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        if constexpr (kSplit) {
            if (fuse_o) {  // waited for before the O rows (every path that issued it reaches that wait)
                mbar_expect_tx(m.bar + 2, ow_bytes);
                bulk_g2s(m.ow, ow_src, ow_bytes, m.bar + 2);
            }
        } else {
            if (fuse_o) l2_prefetch_slice(reinterpret_cast<const char *>(ow_src), ow_bytes, 0, 1);
        }
    }
    __syncthreads();
    // the next kernel (Gate/Up or O) may launch -- and stream its weights on the
    // SMs attention leaves free -- from the start when the context is long, or
    // only once PV is done when it is short: its streaming then slows this
    // kernel's latency-bound loads more than it gains (trigger_tiles, measured)
    const bool early_trigger = st.position + r + 1 > a.trigger_tiles * kTile;
    pdl_wait();
    if (early_trigger) pdl_trigger();
    // every CTA of the cluster reaches every cluster barrier, also when it owns nothing
    const int ctx = st.position + r + 1;
    const int ntiles = row_ok ? (ctx + kTile - 1) / kTile : 0;
    const int tpc = max(1, (ntiles + C - 1) / C);
    const int t_begin = min(c * tpc, ntiles), t_end = min(t_begin + tpc, ntiles);
    const int nown = t_end - t_begin;
    const int p_begin = t_begin * kTile;
    const int npos = nown > 0 ? min(t_end * kTile, ctx) - p_begin : 0;
    const int kvh = (a.first_head + lh) / a.gqa;
    const int16_t *kb = a.kc + ((size_t)kvh * a.max_seq + p_begin) * hd;
    const int16_t *vb = a.vc + ((size_t)kvh * a.max_seq + p_begin) * hd;

    const uint32_t kv_bytes = (uint32_t)npos * hd * 2;
    if (threadIdx.x == 0 && npos > 0) {
        mbar_expect_tx(m.bar, kv_bytes);
        bulk_g2s(m.kv, kb, kv_bytes, m.bar);
    }
    if (npos > 0) {
        const uint4 *qsrc = reinterpret_cast<const uint4 *>(a.q + (size_t)r * a.q_heads * hd + (size_t)lh * hd);
        for (int i = threadIdx.x; i < vpr; i += blockDim.x) reinterpret_cast<uint4 *>(m.q)[i] = qsrc[i];
    }
    for (int i = threadIdx.x; i < nown; i += blockDim.x) m.tsum[i] = 0;
    // L2 warm-up: the same byte count in every CTA (from the step record), one slice each
    const unsigned long long pf_n =
        min(a.pf_bytes, a.pf_per_tile * (unsigned long long)((st.position + st.rows + kTile - 1) / kTile)) & ~15ull;
    if (threadIdx.x == 0 && pf_n && !a.pf_late)
        l2_prefetch_slice(a.pf, pf_n, blockIdx.y * gridDim.x + blockIdx.x, gridDim.x * gridDim.y);
    cp_async_wait_all();
    if (npos > 0 && !mbar_wait(m.bar, 0)) atomicCAS(a.error, 0, kErrAttnCopy);
    __syncthreads();

    // ---- 1. scores; owned tile maxima pushed to every CTA of the cluster ----
    // Banks k mod 4 of golden_attention_mm saturate in k order; a bank holds <= 32
    // products of magnitude <= 2^26 at head_dim <= 128, so no partial sum of <= 31
    // of them leaves int32 and the in-order saturating bank equals sat32 of its
    // exact sum.  Each bank is therefore summed as two exact int32 halves (even /
    // odd 16-byte vectors, <= 16 products each), added in int64 and saturated once.
    const int rot = (threadIdx.x & 31) % vpr;
    for (int pp = threadIdx.x; pp < npos; pp += blockDim.x) {
        const uint4 *qv = reinterpret_cast<const uint4 *>(m.q);
        const uint4 *kv = reinterpret_cast<const uint4 *>(m.kv + pp * hd);
        int32_t b[2][4] = {{0, 0, 0, 0}, {0, 0, 0, 0}};
        auto add8 = [&](int32_t (&c)[4], const uint4 q, const uint4 k) {
            c[0] += qk_prod(lo16(q.x), q412(lo16(k.x)));
            c[1] += qk_prod(hi16(q.x), q412(hi16(k.x)));
            c[2] += qk_prod(lo16(q.y), q412(lo16(k.y)));
            c[3] += qk_prod(hi16(q.y), q412(hi16(k.y)));
            c[0] += qk_prod(lo16(q.z), q412(lo16(k.z)));
            c[1] += qk_prod(hi16(q.z), q412(hi16(k.z)));
            c[2] += qk_prod(lo16(q.w), q412(lo16(k.w)));
            c[3] += qk_prod(hi16(q.w), q412(hi16(k.w)));
        };
        int e8 = 0;
#pragma unroll 2
        for (; e8 + 1 < vpr; e8 += 2) {
            const int v0 = rot_vec(e8 + rot, vpr), v1 = rot_vec(e8 + 1 + rot, vpr);
            add8(b[0], qv[v0], kv[v0]);
            add8(b[1], qv[v1], kv[v1]);
        }
        if (e8 < vpr) {
            const int v0 = rot_vec(e8 + rot, vpr);
            add8(b[0], qv[v0], kv[v0]);
        }
        int64_t t64 = 0;
#pragma unroll
        for (int j = 0; j < 4; j++) t64 += sat32((int64_t)b[0][j] + b[1][j]);
        int32_t tot = sat32(t64);
        tot = sat32(rnd((int64_t)tot * a.qk_scale, 16));  // x accum(fm(1/sqrt(d)))
        const int32_t sc = sat16(rnd(tot, 8));
        m.sc[pp] = (int16_t)sc;
    }
    __syncthreads();  // K consumed: the buffer now receives V (overlaps the exchange below)
    if (threadIdx.x == 0 && npos > 0) {
        mbar_expect_tx(m.bar + 1, kv_bytes);
        bulk_g2s(m.kv, vb, kv_bytes, m.bar + 1);
    }
    {   // tile maxima: one warp per owned tile
        const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
        for (int tl = warp; tl < nown; tl += blockDim.x >> 5) {
            const int pe = min(kTile, npos - tl * kTile);
            int32_t mx = -32768;
            for (int j = lane; j < pe; j += 32) mx = max(mx, (int32_t)m.sc[tl * kTile + j]);
#pragma unroll
            for (int o = 16; o >= 1; o >>= 1) mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, o));
            if (lane < C) *cluster.map_shared_rank(m.mloc + t_begin + tl, lane) = mx;
        }
    }
    cluster.sync();
    if (threadIdx.x == 0 && pf_n && a.pf_late)
        l2_prefetch_slice(a.pf, pf_n, blockIdx.y * gridDim.x + blockIdx.x, gridDim.x * gridDim.y);

    // ---- 2. running maxima, probabilities, tile sums, rescale, PV ----------
    // running max after tile t = prefix max of tile maxima, m_{-1} = fm(-128)
    for (int pp = threadIdx.x; pp < npos; pp += blockDim.x) {
        const int t = t_begin + pp / kTile;
        int32_t mt = -32768;
        for (int u = 0; u <= t; u++) mt = max(mt, m.mloc[u]);
        int32_t d = sat16((int32_t)m.sc[pp] - mt);
        d = d < -2048 ? -2048 : (d > 0 ? 0 : d);
        const int32_t pr = m.ptab[d + 2048];
        m.sc[pp] = (int16_t)pr;
        atomicAdd(m.tsum + pp / kTile, pr * 4);  // Q2.14 -> Q16.16; <= 64 * 2^16, never saturates
    }
    if (npos > 0 && !mbar_wait(m.bar + 1, 0)) atomicCAS(a.error, 0, kErrAttnCopy);
    __syncthreads();
    for (int i = threadIdx.x; i < nown; i += blockDim.x) {  // tile sum + rescale factor -> every CTA
        const int t = t_begin + i;
        int32_t mprev = -32768, mt = -32768;
        for (int u = 0; u < t; u++) mprev = max(mprev, m.mloc[u]);
        mt = max(mprev, m.mloc[t]);
        int32_t d = sat16(mprev - mt);
        d = d < -2048 ? -2048 : d;
        const int32_t old = m.ptab[d + 2048];
        for (int k = 0; k < C; k++) {
            *cluster.map_shared_rank(m.gsum + t, k) = m.tsum[i];
            *cluster.map_shared_rank(m.gold + t, k) = old;
        }
    }
    // raw payload p (read as Q8.8) x V (Q4.12, saturated), rounded per product,
    // four banks in position order (|p*v| <= 2^29: banks never saturate),
    // x accum(fm(1/64)), -> fm; pushed to the CTA that finalises element e
    for (int i = threadIdx.x; i < nown * hd; i += blockDim.x) {
        const int tli = i / hd, e = i - tli * hd;
        const int pb = tli * kTile, pe = min(pb + kTile, npos);
        int32_t b0 = 0, b1 = 0, b2 = 0, b3 = 0;
        int pp = pb;
        for (; pp + 3 < pe; pp += 4) {
            b0 += qk_prod(m.sc[pp], q412(m.kv[pp * hd + e]));
            b1 += qk_prod(m.sc[pp + 1], q412(m.kv[(pp + 1) * hd + e]));
            b2 += qk_prod(m.sc[pp + 2], q412(m.kv[(pp + 2) * hd + e]));
            b3 += qk_prod(m.sc[pp + 3], q412(m.kv[(pp + 3) * hd + e]));
        }
        if (pp < pe) b0 += qk_prod(m.sc[pp], q412(m.kv[pp * hd + e]));
        if (pp + 1 < pe) b1 += qk_prod(m.sc[pp + 1], q412(m.kv[(pp + 1) * hd + e]));
        if (pp + 2 < pe) b2 += qk_prod(m.sc[pp + 2], q412(m.kv[(pp + 2) * hd + e]));
        int32_t ts = sat32((int64_t)b0 + b1 + b2 + b3);
        ts = sat32(rnd((int64_t)ts * 1024, 16));
        const int16_t tv = (int16_t)sat16(rnd(ts, 8));
        if constexpr (kSplit) {  // every CTA runs the whole recurrence
            for (int k = 0; k < C; k++) *cluster.map_shared_rank(m.tvr + (t_begin + tli) * hd + e, k) = tv;
        } else {
            *cluster.map_shared_rank(m.tvr + (t_begin + tli) * epc + e / C, e % C) = tv;
        }
    }
    cluster.sync();
    if (!early_trigger) pdl_trigger();
    if (!kSplit && fuse_o && threadIdx.x == 0) {  // V is consumed: the buffer now receives the O slice
        mbar_expect_tx(m.bar + 2, ow_bytes);
        bulk_g2s(m.ow, ow_src, ow_bytes, m.bar + 2);
    }

    // ---- 3. in-order Q16.16 recurrence on local shared memory ---------------
    if constexpr (kSplit) {  // all hd elements in every CTA (the host launches this variant with o_w only)
        for (int e = threadIdx.x; ntiles > 0 && e < hd; e += blockDim.x) {
            int32_t sum = 0, acc = 0;
            for (int u = 0; u < ntiles; u++) {
                const int64_t o = (int64_t)m.gold[u] * 4;  // Q2.14 -> Q16.16
                sum = sat32(rnd((int64_t)sum * o, 16) + m.gsum[u]);
                acc = sat32(rnd((int64_t)acc * o, 16));
                acc = sat32((int64_t)acc + (int64_t)m.tvr[u * hd + e] * 256);
            }
            const int64_t inv = sat16(rnd((int64_t)recip_q16(sum < 16 ? 16 : sum), 8));
            m.att[e] = (int16_t)sat16(rnd((int64_t)acc * inv * 256, 24));
        }
        __syncthreads();  // after the second cluster barrier no CTA writes another's shared memory
    } else {
        for (int j = threadIdx.x; ntiles > 0 && j < epc; j += blockDim.x) {
            const int e = j * C + c;
            int32_t sum = 0, acc = 0;
            for (int u = 0; u < ntiles; u++) {
                const int64_t o = (int64_t)m.gold[u] * 4;  // Q2.14 -> Q16.16
                sum = sat32(rnd((int64_t)sum * o, 16) + m.gsum[u]);
                acc = sat32(rnd((int64_t)acc * o, 16));
                acc = sat32((int64_t)acc + (int64_t)m.tvr[u * epc + j] * 256);
            }
            const int64_t inv = sat16(rnd((int64_t)recip_q16(sum < 16 ? 16 : sum), 8));
            const int16_t y = (int16_t)sat16(rnd((int64_t)acc * inv * 256, 24));
            if (a.o_w == nullptr) {
                a.out[(size_t)r * a.q_heads * hd + (size_t)lh * hd + e] = y;
            } else {  // the head output -> every CTA of the cluster
                for (int k = 0; k < C; k++) *cluster.map_shared_rank(m.att + e, k) = y;
            }
        }
        if (a.o_w == nullptr) return;
        cluster.sync();
    }

    // ---- 4. fused O projection: this head's exact partial of this CTA's O rows ----
    // (golden_projection host:3105-3142 sums int16 x int16 products exactly and
    // rounds once; the sum over heads is completed by int64 atomics and rounded,
    // with the residual, by the next kernel's prologue)
    if (!fuse_o) return;
    if (!mbar_wait(m.bar + 2, 0)) {
        atomicCAS(a.error, 0, kErrAttnCopy);
        (void)mbar_wait(m.bar + 2, 0);  // give the copies a second bounded wait before leaving
    }
    const uint4 *x4 = reinterpret_cast<const uint4 *>(m.att);
    for (int j = threadIdx.x; j < a.o_rows; j += blockDim.x) {
        const uint4 *w4 = reinterpret_cast<const uint4 *>(m.ow + (size_t)j * (hd >> 1));
        int32_t lo = 0, hi = 0;  // <= 128 products: |lo| < 2^31, |hi| < 2^29
        int v = rot;
        for (int k = 0; k < vpr; k++) {
            const uint4 w = w4[v], x = x4[v];
            lo = dp2a_lo_su(x.x, w.x, lo);
            hi = dp2a_hi_ss(x.x, w.x, hi);
            lo = dp2a_lo_su(x.y, w.y, lo);
            hi = dp2a_hi_ss(x.y, w.y, hi);
            lo = dp2a_lo_su(x.z, w.z, lo);
            hi = dp2a_hi_ss(x.z, w.z, hi);
            lo = dp2a_lo_su(x.w, w.w, lo);
            hi = dp2a_hi_ss(x.w, w.w, hi);
            v = rot_vec(v + 1, vpr);
        }
        const int64_t tot = (int64_t)hi * 256 + lo;
        atomicAdd(reinterpret_cast<unsigned long long *>(a.o_acc + (size_t)r * a.hidden + (size_t)c * a.o_rows + j),
                  (unsigned long long)tot);
    }
    if constexpr (kTp) {
        __shared__ int last_s;
        __syncthreads();  // every atomic of this CTA issued
        if (threadIdx.x == 0) {  // release this CTA's sums / acquire the other heads' (as the stream-K tiles)
            int *cnt = a.o_cnt + r * C + c, old;
            asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], 1;" : "=r"(old) : "l"(cnt) : "memory");
            last_s = old == a.q_heads - 1;
            if (last_s) *cnt = 0;  // next used by the next layer's launch
        }
        __syncthreads();
        if (!last_s) return;
        const uint32_t n = st.ar_base + a.ar_off;
        for (int j = threadIdx.x; j < a.o_rows; j += blockDim.x) {
            const int row = c * a.o_rows + j;
            const int64_t v = (int64_t)atomicExch(
                reinterpret_cast<unsigned long long *>(a.o_acc + (size_t)r * a.hidden + row), 0ull);
            const size_t w = ar_word_index((int)(n & 1u), a.ar.me, r, a.ar.hidden, row);
            const uint64_t word = ar_pack(v, ar_tag(n));
            for (int q = 0; q < a.ar.n; q++) ar_store(reinterpret_cast<uint64_t *>(a.ar.base[q] + kArHeader) + w, word);
        }
    }
}

// ---------------------------------------------------------------------------
// Blocks of several rows: one cluster per query head handles every row of the
// block, so the K and V tiles of the head are read once for all rows.  Row r
// sees positions < position + r + 1 (its own causal context); the cluster's
// tiles cover the longest row.  Per row the arithmetic, the tile order and the
// exchange are those of k_attn above.
// ---------------------------------------------------------------------------
struct AttnRowsSmem {
    int16_t *kv;    // [tpc*64][hd]  K rows, then V rows, shared by the rows
    int16_t *ptab;  // [2049]
    int16_t *q;     // [kMaxRows][hd]
    int16_t *sc;    // [kMaxRows][tpc*64]  scores, then probabilities
    int16_t *tvr;   // [kMaxRows][kMaxTiles][hd/C]
    int32_t *mloc;  // [kMaxRows][kMaxTiles]
    int32_t *gsum;  // [kMaxRows][kMaxTiles]
    int32_t *gold;  // [kMaxRows][kMaxTiles]
    int32_t *tsum;  // [kMaxRows][tpc]
    uint64_t *bar;  // [2] completion of the K and of the V copy
};

static __host__ __device__ size_t attn_rows_layout(int tpc, int cl, size_t off[10]) {
    const size_t P = (size_t)tpc * kTile;
    size_t b = 0;
    off[0] = b; b = align16(b + P * kMaxHd * 2);
    off[1] = b; b = align16(b + kPtabChunks * 16);
    off[2] = b; b = align16(b + (size_t)kMaxRows * kMaxHd * 2);
    off[3] = b; b = align16(b + (size_t)kMaxRows * P * 2);
    off[4] = b; b = align16(b + (size_t)kMaxRows * kMaxTiles * (kMaxHd / cl) * 2);
    off[5] = b; b = align16(b + (size_t)kMaxRows * kMaxTiles * 4);
    off[6] = b; b = align16(b + (size_t)kMaxRows * kMaxTiles * 4);
    off[7] = b; b = align16(b + (size_t)kMaxRows * kMaxTiles * 4);
    off[8] = b; b = align16(b + (size_t)kMaxRows * tpc * 4);
    off[9] = b; b = align16(b + 2 * 8);
    return b;
}

size_t attn_rows_smem_bytes(int tpc, int cluster) {
    size_t off[10];
    return attn_rows_layout(tpc, cluster, off);
}

constexpr int kAttnRowsThreads = 256;
constexpr int kRowGroup = 4;  // rows per thread in the row-inner loop order

// kRowInner (LLMX_ATTN_ROWS_INNER): QK and PV loop over a group of kRowGroup
// rows innermost, so each K / V element is converted to Q4.12 and each K vector
// loaded once per group instead of once per row.  The products, their banks
// (element index mod 4 for QK, position mod 4 for PV) and the halves are those
// of the row-outer order, so every sum is the same exact integer.
template <int C, bool kRowInner>
__global__ void __launch_bounds__(kAttnRowsThreads) k_attn_rows(const AttnArgs a) {
    LLMX_TL_GUARD(a.tl_slot);
    extern __shared__ __align__(16) char raw[];
    cg::cluster_group cluster = cg::this_cluster();
    const int c = (int)cluster.block_rank();
    const int lh = blockIdx.x / C;
    const int hd = a.hd, vpr = hd >> 3, epc = hd / C;
    size_t off[10];
    attn_rows_layout(a.tpc_max, C, off);
    AttnRowsSmem m;
    m.kv = reinterpret_cast<int16_t *>(raw + off[0]);
    m.ptab = reinterpret_cast<int16_t *>(raw + off[1]);
    m.q = reinterpret_cast<int16_t *>(raw + off[2]);
    m.sc = reinterpret_cast<int16_t *>(raw + off[3]);
    m.tvr = reinterpret_cast<int16_t *>(raw + off[4]);
    m.mloc = reinterpret_cast<int32_t *>(raw + off[5]);
    m.gsum = reinterpret_cast<int32_t *>(raw + off[6]);
    m.gold = reinterpret_cast<int32_t *>(raw + off[7]);
    m.tsum = reinterpret_cast<int32_t *>(raw + off[8]);
    m.bar = reinterpret_cast<uint64_t *>(raw + off[9]);
    const int P = a.tpc_max * kTile;  // row stride of sc

    for (int i = threadIdx.x; i < kPtabChunks; i += blockDim.x) cp_async16(m.ptab + 8 * i, a.ptab + 8 * i);
    if (threadIdx.x == 0) {
        mbar_init(m.bar, 1);
        mbar_init(m.bar + 1, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    const Step st = load_step(a.step);
    __syncthreads();
    pdl_wait();
    pdl_trigger();  // a block's next kernel may launch at once (a later trigger measured slower here)
    const int R = st.rows;
    const int ntiles = (st.position + R + kTile - 1) / kTile;  // the longest row's tiles
    const int tpc = max(1, (ntiles + C - 1) / C);
    const int t_begin = min(c * tpc, ntiles), t_end = min(t_begin + tpc, ntiles);
    const int nown = t_end - t_begin;
    const int p_begin = t_begin * kTile;
    const int npos = nown > 0 ? min(t_end * kTile, st.position + R) - p_begin : 0;
    auto npos_of = [&](int r) { return max(0, min(npos, st.position + r + 1 - p_begin)); };
    auto ntiles_of = [&](int r) { return (st.position + r + 1 + kTile - 1) / kTile; };
    const int kvh = (a.first_head + lh) / a.gqa;
    const int16_t *kb = a.kc + ((size_t)kvh * a.max_seq + p_begin) * hd;
    const int16_t *vb = a.vc + ((size_t)kvh * a.max_seq + p_begin) * hd;

    const uint32_t kv_bytes = (uint32_t)npos * hd * 2;
    if (threadIdx.x == 0 && npos > 0) {
        mbar_expect_tx(m.bar, kv_bytes);
        bulk_g2s(m.kv, kb, kv_bytes, m.bar);
    }
    for (int i = threadIdx.x; i < R * vpr; i += blockDim.x) {
        const int r = i / vpr, v = i - r * vpr;
        reinterpret_cast<uint4 *>(m.q + r * kMaxHd)[v] =
            reinterpret_cast<const uint4 *>(a.q + (size_t)r * a.q_heads * hd + (size_t)lh * hd)[v];
    }
    for (int i = threadIdx.x; i < R * tpc; i += blockDim.x) m.tsum[i] = 0;
    cp_async_wait_all();
    if (npos > 0 && !mbar_wait(m.bar, 0)) atomicCAS(a.error, 0, kErrAttnCopy);
    __syncthreads();

    // ---- 1. scores of every (row, position) of the row's context -----------
    const int rot = (threadIdx.x & 31) % vpr;
    if constexpr (kRowInner) {
        const int groups = (R + kRowGroup - 1) / kRowGroup;
        for (int i = threadIdx.x; i < groups * npos; i += blockDim.x) {
            const int g = i / npos, pp = i - g * npos, r0 = g * kRowGroup;
            const uint4 *kv = reinterpret_cast<const uint4 *>(m.kv + pp * hd);
            int32_t b[kRowGroup][2][4];
#pragma unroll
            for (int rr = 0; rr < kRowGroup; rr++)
#pragma unroll
                for (int j = 0; j < 4; j++) b[rr][0][j] = b[rr][1][j] = 0;
            for (int e8 = 0; e8 < vpr; e8 += 2) {
#pragma unroll
                for (int h = 0; h < 2; h++) {  // half h: the row-outer loop's b[h] (vectors e8 + h)
                    if (e8 + h >= vpr) break;
                    const int v = rot_vec(e8 + h + rot, vpr);
                    const uint4 k = kv[v];
                    const int32_t kk[8] = {q412(lo16(k.x)), q412(hi16(k.x)), q412(lo16(k.y)), q412(hi16(k.y)),
                                           q412(lo16(k.z)), q412(hi16(k.z)), q412(lo16(k.w)), q412(hi16(k.w))};
#pragma unroll
                    for (int rr = 0; rr < kRowGroup; rr++) {
                        const uint4 q = reinterpret_cast<const uint4 *>(m.q + (r0 + rr) * kMaxHd)[v];
                        b[rr][h][0] += qk_prod(lo16(q.x), kk[0]);
                        b[rr][h][1] += qk_prod(hi16(q.x), kk[1]);
                        b[rr][h][2] += qk_prod(lo16(q.y), kk[2]);
                        b[rr][h][3] += qk_prod(hi16(q.y), kk[3]);
                        b[rr][h][0] += qk_prod(lo16(q.z), kk[4]);
                        b[rr][h][1] += qk_prod(hi16(q.z), kk[5]);
                        b[rr][h][2] += qk_prod(lo16(q.w), kk[6]);
                        b[rr][h][3] += qk_prod(hi16(q.w), kk[7]);
                    }
                }
            }
#pragma unroll
            for (int rr = 0; rr < kRowGroup; rr++) {
                const int r = r0 + rr;
                if (r >= R || pp >= npos_of(r)) continue;  // rows past the block: garbage q, never stored
                int64_t t64 = 0;
#pragma unroll
                for (int j = 0; j < 4; j++) t64 += sat32((int64_t)b[rr][0][j] + b[rr][1][j]);
                int32_t tot = sat32(t64);
                tot = sat32(rnd((int64_t)tot * a.qk_scale, 16));
                m.sc[r * P + pp] = (int16_t)sat16(rnd(tot, 8));
            }
        }
    } else
    for (int i = threadIdx.x; i < R * npos; i += blockDim.x) {
        const int r = i / npos, pp = i - r * npos;
        if (pp >= npos_of(r)) continue;
        const uint4 *qv = reinterpret_cast<const uint4 *>(m.q + r * kMaxHd);
        const uint4 *kv = reinterpret_cast<const uint4 *>(m.kv + pp * hd);
        int32_t b[2][4] = {{0, 0, 0, 0}, {0, 0, 0, 0}};
        auto add8 = [&](int32_t (&cc)[4], const uint4 q, const uint4 k) {
            cc[0] += qk_prod(lo16(q.x), q412(lo16(k.x)));
            cc[1] += qk_prod(hi16(q.x), q412(hi16(k.x)));
            cc[2] += qk_prod(lo16(q.y), q412(lo16(k.y)));
            cc[3] += qk_prod(hi16(q.y), q412(hi16(k.y)));
            cc[0] += qk_prod(lo16(q.z), q412(lo16(k.z)));
            cc[1] += qk_prod(hi16(q.z), q412(hi16(k.z)));
            cc[2] += qk_prod(lo16(q.w), q412(lo16(k.w)));
            cc[3] += qk_prod(hi16(q.w), q412(hi16(k.w)));
        };
        int e8 = 0;
        for (; e8 + 1 < vpr; e8 += 2) {
            const int v0 = rot_vec(e8 + rot, vpr), v1 = rot_vec(e8 + 1 + rot, vpr);
            add8(b[0], qv[v0], kv[v0]);
            add8(b[1], qv[v1], kv[v1]);
        }
        if (e8 < vpr) {
            const int v0 = rot_vec(e8 + rot, vpr);
            add8(b[0], qv[v0], kv[v0]);
        }
        int64_t t64 = 0;
#pragma unroll
        for (int j = 0; j < 4; j++) t64 += sat32((int64_t)b[0][j] + b[1][j]);
        int32_t tot = sat32(t64);
        tot = sat32(rnd((int64_t)tot * a.qk_scale, 16));
        m.sc[r * P + pp] = (int16_t)sat16(rnd(tot, 8));
    }
    __syncthreads();  // K consumed: the buffer now receives V
    if (threadIdx.x == 0 && npos > 0) {
        mbar_expect_tx(m.bar + 1, kv_bytes);
        bulk_g2s(m.kv, vb, kv_bytes, m.bar + 1);
    }
    {   // tile maxima of every (row, owned tile in the row's context): one warp each
        const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
        for (int w = warp; w < R * nown; w += blockDim.x >> 5) {
            const int r = w / nown, tl = w - r * nown;
            const int pe = min(kTile, npos_of(r) - tl * kTile);
            if (pe <= 0) continue;
            int32_t mx = -32768;
            for (int j = lane; j < pe; j += 32) mx = max(mx, (int32_t)m.sc[r * P + tl * kTile + j]);
#pragma unroll
            for (int o = 16; o >= 1; o >>= 1) mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, o));
            if (lane < C) *cluster.map_shared_rank(m.mloc + r * kMaxTiles + t_begin + tl, lane) = mx;
        }
    }
    cluster.sync();

    // ---- 2. probabilities, tile sums and rescale factors, PV ----------------
    for (int i = threadIdx.x; i < R * npos; i += blockDim.x) {
        const int r = i / npos, pp = i - r * npos;
        if (pp >= npos_of(r)) continue;
        const int t = t_begin + pp / kTile;
        const int32_t *ml = m.mloc + r * kMaxTiles;
        int32_t mt = -32768;
        for (int u = 0; u <= t; u++) mt = max(mt, ml[u]);
        int32_t d = sat16((int32_t)m.sc[r * P + pp] - mt);
        d = d < -2048 ? -2048 : (d > 0 ? 0 : d);
        const int32_t pr = m.ptab[d + 2048];
        m.sc[r * P + pp] = (int16_t)pr;
        atomicAdd(m.tsum + r * tpc + pp / kTile, pr * 4);
    }
    if (npos > 0 && !mbar_wait(m.bar + 1, 0)) atomicCAS(a.error, 0, kErrAttnCopy);
    __syncthreads();
    for (int i = threadIdx.x; i < R * nown; i += blockDim.x) {
        const int r = i / nown, tl = i - r * nown, t = t_begin + tl;
        if (t >= ntiles_of(r)) continue;
        const int32_t *ml = m.mloc + r * kMaxTiles;
        int32_t mprev = -32768;
        for (int u = 0; u < t; u++) mprev = max(mprev, ml[u]);
        const int32_t mt = max(mprev, ml[t]);
        int32_t d = sat16(mprev - mt);
        d = d < -2048 ? -2048 : d;
        const int32_t old = m.ptab[d + 2048];
        for (int k = 0; k < C; k++) {
            *cluster.map_shared_rank(m.gsum + r * kMaxTiles + t, k) = m.tsum[r * tpc + tl];
            *cluster.map_shared_rank(m.gold + r * kMaxTiles + t, k) = old;
        }
    }
    if constexpr (kRowInner) {
        const int groups = (R + kRowGroup - 1) / kRowGroup;
        for (int i = threadIdx.x; i < groups * nown * hd; i += blockDim.x) {
            const int g = i / (nown * hd), rem = i - g * nown * hd, tli = rem / hd, e = rem - tli * hd;
            const int r0 = g * kRowGroup, pb = tli * kTile;
            int pe_r[kRowGroup], pe_max = pb;
#pragma unroll
            for (int rr = 0; rr < kRowGroup; rr++) {  // end of this tile in row r0 + rr's context
                pe_r[rr] = r0 + rr < R ? min(pb + kTile, npos_of(r0 + rr)) : pb;
                pe_max = max(pe_max, pe_r[rr]);
            }
            if (pe_max <= pb) continue;
            int32_t bk[kRowGroup][4];
#pragma unroll
            for (int rr = 0; rr < kRowGroup; rr++)
#pragma unroll
                for (int j = 0; j < 4; j++) bk[rr][j] = 0;
            for (int p4 = pb; p4 < pe_max; p4 += 4) {
#pragma unroll
                for (int j = 0; j < 4; j++) {  // bank j: positions pb + j (mod 4), as in the row-outer loop
                    const int pp = p4 + j;
                    if (pp >= pe_max) break;
                    const int32_t vv = q412(m.kv[pp * hd + e]);
#pragma unroll
                    for (int rr = 0; rr < kRowGroup; rr++)
                        if (pp < pe_r[rr]) bk[rr][j] += qk_prod(m.sc[(r0 + rr) * P + pp], vv);
                }
            }
#pragma unroll
            for (int rr = 0; rr < kRowGroup; rr++) {
                const int r = r0 + rr;
                if (pe_r[rr] <= pb) continue;  // past the block, or the tile is beyond this row's context
                int32_t ts = sat32((int64_t)bk[rr][0] + bk[rr][1] + bk[rr][2] + bk[rr][3]);
                ts = sat32(rnd((int64_t)ts * 1024, 16));
                const int16_t tv = (int16_t)sat16(rnd(ts, 8));
                *cluster.map_shared_rank(m.tvr + (r * kMaxTiles + t_begin + tli) * epc + e / C, e % C) = tv;
            }
        }
    } else
    for (int i = threadIdx.x; i < R * nown * hd; i += blockDim.x) {
        const int r = i / (nown * hd), rem = i - r * nown * hd, tli = rem / hd, e = rem - tli * hd;
        const int pb = tli * kTile, pe = min(pb + kTile, npos_of(r));
        if (pe <= pb) continue;
        const int16_t *scr = m.sc + r * P;
        int32_t b0 = 0, b1 = 0, b2 = 0, b3 = 0;
        int pp = pb;
        for (; pp + 3 < pe; pp += 4) {
            b0 += qk_prod(scr[pp], q412(m.kv[pp * hd + e]));
            b1 += qk_prod(scr[pp + 1], q412(m.kv[(pp + 1) * hd + e]));
            b2 += qk_prod(scr[pp + 2], q412(m.kv[(pp + 2) * hd + e]));
            b3 += qk_prod(scr[pp + 3], q412(m.kv[(pp + 3) * hd + e]));
        }
        if (pp < pe) b0 += qk_prod(scr[pp], q412(m.kv[pp * hd + e]));
        if (pp + 1 < pe) b1 += qk_prod(scr[pp + 1], q412(m.kv[(pp + 1) * hd + e]));
        if (pp + 2 < pe) b2 += qk_prod(scr[pp + 2], q412(m.kv[(pp + 2) * hd + e]));
        int32_t ts = sat32((int64_t)b0 + b1 + b2 + b3);
        ts = sat32(rnd((int64_t)ts * 1024, 16));
        const int16_t tv = (int16_t)sat16(rnd(ts, 8));
        *cluster.map_shared_rank(m.tvr + (r * kMaxTiles + t_begin + tli) * epc + e / C, e % C) = tv;
    }
    cluster.sync();

    // ---- 3. in-order Q16.16 recurrence per row ------------------------------
    for (int i = threadIdx.x; i < R * epc; i += blockDim.x) {
        const int r = i / epc, j = i - r * epc, e = j * C + c;
        const int nt = ntiles_of(r);
        int32_t sum = 0, acc = 0;
        for (int u = 0; u < nt; u++) {
            const int64_t o = (int64_t)m.gold[r * kMaxTiles + u] * 4;
            sum = sat32(rnd((int64_t)sum * o, 16) + m.gsum[r * kMaxTiles + u]);
            acc = sat32(rnd((int64_t)acc * o, 16));
            acc = sat32((int64_t)acc + (int64_t)m.tvr[(r * kMaxTiles + u) * epc + j] * 256);
        }
        const int64_t inv = sat16(rnd((int64_t)recip_q16(sum < 16 ? 16 : sum), 8));
        a.out[(size_t)r * a.q_heads * hd + (size_t)lh * hd + e] = (int16_t)sat16(rnd((int64_t)acc * inv * 256, 24));
    }
}

template <bool kRowInner>
static cudaError_t attn_rows_configure_v(int max_smem_bytes, int cluster) {
    if (cluster == kClusterWide) {
        cudaError_t e = cudaFuncSetAttribute(k_attn_rows<kClusterWide, kRowInner>,
                                             cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
        if (e != cudaSuccess) return e;
        return cudaFuncSetAttribute(k_attn_rows<kClusterWide, kRowInner>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    max_smem_bytes);
    }
    return cudaFuncSetAttribute(k_attn_rows<kCluster, kRowInner>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                max_smem_bytes);
}

cudaError_t attn_rows_configure(int max_smem_bytes, int cluster) {
    cudaError_t e = attn_rows_configure_v<false>(max_smem_bytes, cluster);
    if (e != cudaSuccess) return e;
    return attn_rows_configure_v<true>(max_smem_bytes, cluster);
}

cudaError_t launch_attn_rows(const AttnArgs &a, cudaStream_t s) {
    AttnArgs c = a;
    LLMX_TL_TAKE(c, "attn_rows");
    void *args[] = {&c};
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.cluster * a.q_heads, 1);
    cfg.blockDim = dim3(kAttnRowsThreads);
    cfg.dynamicSmemBytes = attn_rows_smem_bytes(a.tpc_max, a.cluster);
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = a.cluster;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    const bool wide = a.cluster == kClusterWide;
    const void *fn = a.rows_inner ? (wide ? (const void *)k_attn_rows<kClusterWide, true>
                                          : (const void *)k_attn_rows<kCluster, true>)
                                  : (wide ? (const void *)k_attn_rows<kClusterWide, false>
                                          : (const void *)k_attn_rows<kCluster, false>);
    return cudaLaunchKernelExC(&cfg, fn, args);
}

template <bool kTp>
static cudaError_t attn_configure_v(int max_smem_bytes, int cluster) {
    if (cluster == kClusterWide) {
        cudaError_t e =
            cudaFuncSetAttribute(k_attn<kClusterWide, false, kTp>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
        if (e != cudaSuccess) return e;
        return cudaFuncSetAttribute(k_attn<kClusterWide, false, kTp>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    max_smem_bytes);
    }
    return cudaFuncSetAttribute(k_attn<kCluster, false, kTp>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                max_smem_bytes);
}

cudaError_t attn_configure(int max_smem_bytes, int cluster, bool tp) {
    cudaError_t e = attn_configure_v<false>(max_smem_bytes, cluster);
    if (e == cudaSuccess && tp) e = attn_configure_v<true>(max_smem_bytes, cluster);
    return e;
}

cudaError_t attn_split_configure(int smem_bytes, int q_heads, int *ok) {
    *ok = 0;
    cudaError_t e =
        cudaFuncSetAttribute(k_attn<kCluster, true, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes);
    if (e != cudaSuccess) return e;
    // every cluster of the one-row grid must be resident at once
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(kCluster * q_heads, 1);
    cfg.blockDim = dim3(kAttnThreads);
    cfg.dynamicSmemBytes = smem_bytes;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = kCluster;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int clusters = 0;
    e = cudaOccupancyMaxActiveClusters(&clusters, (const void *)k_attn<kCluster, true, false>, &cfg);
    if (e != cudaSuccess) return e;
    *ok = clusters >= q_heads ? 1 : 0;
    return cudaSuccess;
}

cudaError_t launch_attn(const AttnArgs &a, int rows, cudaStream_t s) {
    AttnArgs c = a;
    LLMX_TL_TAKE(c, a.o_w != nullptr ? "attn+o" : "attn");
    void *args[] = {&c};
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.cluster * a.q_heads, rows);
    cfg.blockDim = dim3(kAttnThreads);
    // the push to the peers only with the fused O projection on a tensor-parallel
    // rank; the split variant only for the fused O projection of one GPU on 8-CTA clusters
    const bool tp = a.o_w != nullptr && a.ar.n > 1;
    const bool split = !tp && a.split_o && a.o_w != nullptr && a.cluster == kCluster;
    cfg.dynamicSmemBytes = attn_smem_bytes(a.tpc_max, a.hd, a.cluster, a.o_w != nullptr ? a.o_rows : 0, split);
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = a.cluster;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    const bool wide = a.cluster == kClusterWide;
    const void *fn = tp      ? (wide ? (const void *)k_attn<kClusterWide, false, true>
                                     : (const void *)k_attn<kCluster, false, true>)
                     : wide  ? (const void *)k_attn<kClusterWide, false, false>
                     : split ? (const void *)k_attn<kCluster, true, false>
                             : (const void *)k_attn<kCluster, false, false>;
    return cudaLaunchKernelExC(&cfg, fn, args);
}

}  // namespace llmx

LLMX_TL_READER(attention)
