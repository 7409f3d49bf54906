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

namespace llmx {

namespace cg = cooperative_groups;

constexpr int kKvStride = 136;  // padded smem row (int16): 272 B, 16-B aligned, conflict-free LDS.128
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

// ---- exact fast forms of the per-product rounding ---------------------------
// qk_prod(x, q412(y)) = (x * sat16(16 y) + 8) >> 4 is exactly x * y for
// -2048 <= y <= 2047 (16 y is a multiple of 16 and in range) and x * -2048 for
// y < -2048; only y >= 2048 (sat16(16 y) = 32767) differs from
// x * clamp(y, -2048, 2047).  The kernels clamp K and V to [-2048, 2047] in
// shared memory and form plain integer products -- QK on the dp2a pipe with the
// query split into bytes, PV as 32-bit multiply-adds -- and route every
// position (QK) or tile (PV) that held a y >= 2048, and every query holding
// -32768, through the per-product form again (rare in practice; exact always).
// Without those, no product reaches 2^26 in magnitude, so no bank of <= 32
// products saturates and the sum over all banks equals the banked sum.

// Clamps the 8 int16 of v to [-2048, 2047]; true if one of them was >= 2048.
static __device__ __forceinline__ bool clamp_k12(uint4 &v) {
    uint32_t w[4] = {v.x, v.y, v.z, v.w};
    uint32_t sat = 0;
#pragma unroll
    for (int q = 0; q < 4; q++) {
        sat |= __vcmpges2(w[q], 0x08000800u);
        w[q] = __vmaxs2(__vmins2(w[q], 0x07FF07FFu), 0xF800F800u);
    }
    v = make_uint4(w[0], w[1], w[2], w[3]);
    return sat != 0;
}
// A packed pair of query elements as dp2a operand bytes {lo q0, lo q1, hi q0, hi q1}.
static __device__ __forceinline__ uint32_t q_pair_bytes(uint32_t w) { return __byte_perm(w, 0, 0x3120); }
// QK of one position from clamped K (int16 pairs) and query bytes: exact sum of q * k.
static __device__ __forceinline__ int32_t qk_dot_fast(const uint4 *__restrict__ k, const uint4 *__restrict__ qb,
                                                      int vpr) {
    int lo = 0, hi = 0;
    for (int v = 0; v < vpr; v++) {
        const uint4 kv = k[v], b = qb[v];
        lo = dp2a_lo_su(kv.x, b.x, lo);
        hi = dp2a_hi_ss(kv.x, b.x, hi);
        lo = dp2a_lo_su(kv.y, b.y, lo);
        hi = dp2a_hi_ss(kv.y, b.y, hi);
        lo = dp2a_lo_su(kv.z, b.z, lo);
        hi = dp2a_hi_ss(kv.z, b.z, hi);
        lo = dp2a_lo_su(kv.w, b.w, lo);
        hi = dp2a_hi_ss(kv.w, b.w, hi);
    }
    return sat32((int64_t)lo + 256 * (int64_t)hi);
}
// QK of one position by the per-product rounding, four saturating banks (k mod 4)
// (golden_attention_mm host:3231-3276), from the unclamped rows in global memory.
static __device__ int32_t qk_dot_exact(const int16_t *__restrict__ q, const int16_t *__restrict__ k, int hd) {
    int64_t bank[4] = {0, 0, 0, 0};  // <= 32 products each: the saturating sum is sat32 of the exact one
    for (int i = 0; i < hd; i++) bank[i & 3] += qk_prod(q[i], q412(k[i]));
    int64_t t = 0;
#pragma unroll
    for (int j = 0; j < 4; j++) t += sat32(bank[j]);
    return sat32(t);
}
// Raw-payload PV of one element over positions [0, n) by the per-product rounding,
// from the unclamped V rows in global memory (banks never saturate).
static __device__ int32_t pv_exact(const int16_t *__restrict__ p, const int16_t *__restrict__ v, int hd, int n) {
    int64_t s = 0;
    for (int pp = 0; pp < n; pp++) s += qk_prod(p[pp], q412(v[(size_t)pp * hd]));
    return sat32(s);
}

struct AttnSmem {      // carved out of dynamic shared memory
    int16_t *kv;       // [tpc*64][kKvStride] raw Q8.8 K rows, then V rows, of the owned tiles
    int16_t *ptab;     // [2049] softmax exp table
    int16_t *q;        // [hd]
    int16_t *sc;       // [tpc*64] scores, then Q2.14 probabilities
    int16_t *tvr;      // [kMaxTiles][hd/C] tile values of the elements this CTA finalises
    int32_t *mloc;     // [kMaxTiles] every tile's maximum (pushed by the owners)
    int32_t *gsum;     // [kMaxTiles] every tile's sum (pushed)
    int32_t *gold;     // [kMaxTiles] every tile's rescale factor (pushed)
    int32_t *tsum;     // [tpc] owned tile sums (local accumulation)
    uint32_t *qb;      // [hd/2] query pairs as dp2a bytes
    uint8_t *ksat;     // [tpc*64] position holds a k >= 2048 (exact path)
    int32_t *vsat;     // [tpc] owned tile holds a v >= 2048 (exact path); [tpc] = query holds -32768
};

static __host__ __device__ size_t align16(size_t b) { return (b + 15) & ~size_t(15); }

static __host__ __device__ size_t attn_layout(int tpc, int hd, int cl, size_t off[12]) {
    const size_t rows = (size_t)tpc * kTile;
    size_t b = 0;
    off[0] = b; b = align16(b + rows * kKvStride * 2);                       // kv
    off[1] = b; b = align16(b + 2049 * 2);                                   // ptab
    off[2] = b; b = align16(b + (size_t)kMaxHd * 2);                         // q
    off[3] = b; b = align16(b + rows * 2);                                   // sc
    off[4] = b; b = align16(b + (size_t)kMaxTiles * (kMaxHd / cl) * 2);      // tvr
    off[5] = b; b = align16(b + (size_t)kMaxTiles * 4);                      // mloc
    off[6] = b; b = align16(b + (size_t)kMaxTiles * 4);                      // gsum
    off[7] = b; b = align16(b + (size_t)kMaxTiles * 4);                      // gold
    off[8] = b; b = align16(b + (size_t)tpc * 4);                            // tsum
    off[9] = b; b = align16(b + (size_t)kMaxHd * 2);                         // qb
    off[10] = b; b = align16(b + rows);                                      // ksat
    off[11] = b; b = align16(b + (size_t)(tpc + 1) * 4);                     // vsat + query flag
    (void)hd;
    return b;
}

size_t attn_smem_bytes(int tpc, int hd, int cluster) {
    size_t off[12];
    return attn_layout(tpc, hd, cluster, off);
}


template <int C>
__global__ void __launch_bounds__(kAttnThreads) k_attn(const AttnArgs a) {
    extern __shared__ __align__(16) char raw[];
    cg::cluster_group cluster = cg::this_cluster();
    const int c = (int)cluster.block_rank();
    const int lh = blockIdx.x / C;  // local query head
    const int r = blockIdx.y;
    const int hd = a.hd, vpr = hd >> 3, epc = hd / C;  // elements finalised per CTA
    size_t off[12];
    attn_layout(a.tpc_max, hd, C, off);
    AttnSmem m;
    m.qb = reinterpret_cast<uint32_t *>(raw + off[9]);
    m.ksat = reinterpret_cast<uint8_t *>(raw + off[10]);
    m.vsat = reinterpret_cast<int32_t *>(raw + off[11]);
    m.kv = reinterpret_cast<int16_t *>(raw + off[0]);
    m.ptab = reinterpret_cast<int16_t *>(raw + off[1]);
    m.q = reinterpret_cast<int16_t *>(raw + off[2]);
    m.sc = reinterpret_cast<int16_t *>(raw + off[3]);
    m.tvr = reinterpret_cast<int16_t *>(raw + off[4]);
    m.mloc = reinterpret_cast<int32_t *>(raw + off[5]);
    m.gsum = reinterpret_cast<int32_t *>(raw + off[6]);
    m.gold = reinterpret_cast<int32_t *>(raw + off[7]);
    m.tsum = reinterpret_cast<int32_t *>(raw + off[8]);

    // the exp table does not depend on the producer kernel
    for (int i = threadIdx.x; i < 2049; i += blockDim.x) m.ptab[i] = a.ptab[i];
    pdl_wait();
    pdl_trigger();
    const Step st = *a.step;
    // every CTA of the cluster reaches both cluster barriers, also when it owns nothing
    const bool row_ok = r < st.rows;
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

    for (int i = threadIdx.x; i < npos * vpr; i += blockDim.x) {
        const int pp = i / vpr, cc = (i - pp * vpr) << 3;
        cp_async16(m.kv + pp * kKvStride + cc, kb + (size_t)pp * hd + cc);
    }
    if (npos > 0) {
        const uint4 *qsrc = reinterpret_cast<const uint4 *>(a.q + (size_t)r * a.q_heads * hd + (size_t)lh * hd);
        for (int i = threadIdx.x; i < vpr; i += blockDim.x) reinterpret_cast<uint4 *>(m.q)[i] = qsrc[i];
    }
    for (int i = threadIdx.x; i < nown; i += blockDim.x) m.tsum[i] = 0;
    for (int i = threadIdx.x; i < npos; i += blockDim.x) m.ksat[i] = 0;
    for (int i = threadIdx.x; i <= tpc; i += blockDim.x) m.vsat[i] = 0;
    // L2 warm-up: the same byte count in every CTA (from the step record), one slice each
    const unsigned long long pf_n =
        min(a.pf_bytes, a.pf_per_tile * (unsigned long long)((st.position + st.rows + kTile - 1) / kTile)) & ~15ull;
    if (threadIdx.x == 0 && pf_n && !a.pf_late)
        l2_prefetch_slice(a.pf, pf_n, blockIdx.y * gridDim.x + blockIdx.x, gridDim.x * gridDim.y);
    cp_async_wait_all();
    __syncthreads();
    // clamp K in place (flagging positions with a k >= 2048); query -> dp2a bytes
    const int16_t *qg = a.q + (size_t)r * a.q_heads * hd + (size_t)lh * hd;
    for (int i = threadIdx.x; i < npos * vpr; i += blockDim.x) {
        const int pp = i / vpr, cc = (i - pp * vpr) << 3;
        uint4 *kp = reinterpret_cast<uint4 *>(m.kv + pp * kKvStride + cc);
        uint4 kv = *kp;
        if (clamp_k12(kv)) m.ksat[pp] = 1;
        *kp = kv;
    }
    for (int i = threadIdx.x; npos > 0 && i < vpr; i += blockDim.x) {
        const uint4 qv = reinterpret_cast<const uint4 *>(m.q)[i];
        if ((__vcmpeq2(qv.x, 0x80008000u) | __vcmpeq2(qv.y, 0x80008000u) | __vcmpeq2(qv.z, 0x80008000u) |
             __vcmpeq2(qv.w, 0x80008000u)) != 0)
            m.vsat[tpc] = 1;
        reinterpret_cast<uint4 *>(m.qb)[i] =
            make_uint4(q_pair_bytes(qv.x), q_pair_bytes(qv.y), q_pair_bytes(qv.z), q_pair_bytes(qv.w));
    }
    __syncthreads();
    const bool q_min = m.vsat[tpc] != 0;

    // ---- 1. scores; owned tile maxima pushed to every CTA of the cluster ----
    // Banks k mod 4 of golden_attention_mm saturate in k order; a bank holds <= 32
    // products of magnitude <= 2^26 at head_dim <= 128, so no partial sum of <= 31
    // of them leaves int32 and the in-order saturating bank equals sat32 of its
    // exact sum.  Each bank is therefore summed as two exact int32 halves (even /
    // odd 16-byte vectors, <= 16 products each), added in int64 and saturated once.
    for (int pp = threadIdx.x; pp < npos; pp += blockDim.x) {
        int32_t tot = m.ksat[pp] || q_min ? qk_dot_exact(qg, kb + (size_t)pp * hd, hd)
                                          : qk_dot_fast(reinterpret_cast<const uint4 *>(m.kv + pp * kKvStride),
                                                        reinterpret_cast<const uint4 *>(m.qb), vpr);
        tot = sat32(rnd((int64_t)tot * a.qk_scale, 16));  // x accum(fm(1/sqrt(d)))
        m.sc[pp] = (int16_t)sat16(rnd(tot, 8));
    }
    __syncthreads();  // K consumed: the buffer now receives V (overlaps the exchange below)
    for (int i = threadIdx.x; i < npos * vpr; i += blockDim.x) {
        const int pp = i / vpr, cc = (i - pp * vpr) << 3;
        cp_async16(m.kv + pp * kKvStride + cc, vb + (size_t)pp * hd + cc);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
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
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    __syncthreads();
    for (int i = threadIdx.x; i < npos * vpr; i += blockDim.x) {  // clamp V in place, flag tiles with v >= 2048
        const int pp = i / vpr, cc = (i - pp * vpr) << 3;
        uint4 *vp = reinterpret_cast<uint4 *>(m.kv + pp * kKvStride + cc);
        uint4 vv = *vp;
        if (clamp_k12(vv)) m.vsat[pp / kTile] = 1;
        *vp = vv;
    }
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
    __syncthreads();  // V clamped and tiles flagged
    // raw payload p (read as Q8.8) x V (Q4.12, saturated), rounded per product,
    // four banks in position order (|p*v| <= 2^29: banks never saturate, so
    // their sum is one exact sum), x accum(fm(1/64)), -> fm; pushed to the CTA
    // that finalises element e.  One pair of elements per item.
    for (int i = threadIdx.x; i < nown * (hd >> 1); i += blockDim.x) {
        const int tli = i / (hd >> 1), e = 2 * (i - tli * (hd >> 1));
        const int pb = tli * kTile, pe = min(pb + kTile, npos);
        int32_t s2[2];
        if (m.vsat[tli]) {
            s2[0] = pv_exact(m.sc + pb, vb + (size_t)pb * hd + e, hd, pe - pb);
            s2[1] = pv_exact(m.sc + pb, vb + (size_t)pb * hd + e + 1, hd, pe - pb);
        } else {  // |p * v| <= 2^14 * 2^11: 64 products stay within int32
            int32_t a0 = 0, a1 = 0;
            for (int pp = pb; pp < pe; pp++) {
                const int32_t pr = m.sc[pp];
                const uint32_t w = *reinterpret_cast<const uint32_t *>(m.kv + pp * kKvStride + e);
                a0 += pr * lo16(w);
                a1 += pr * hi16(w);
            }
            s2[0] = a0;
            s2[1] = a1;
        }
#pragma unroll
        for (int h = 0; h < 2; h++) {
            const int32_t ts = sat32(rnd((int64_t)s2[h] * 1024, 16));
            const int16_t tv = (int16_t)sat16(rnd(ts, 8));
            *cluster.map_shared_rank(m.tvr + (t_begin + tli) * epc + (e + h) / C, (e + h) % C) = tv;
        }
    }
    cluster.sync();

    // ---- 3. in-order Q16.16 recurrence on local shared memory ---------------
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
        a.out[(size_t)r * a.q_heads * hd + (size_t)lh * hd + e] = (int16_t)sat16(rnd((int64_t)acc * inv * 256, 24));
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
    int16_t *kv;    // [tpc*64][kKvStride]  K rows, then V rows, shared by the rows
    int16_t *ptab;  // [2049]
    int16_t *q;     // [kMaxRows][hd]
    int16_t *sc;    // [kMaxRows][tpc*64]  scores, then probabilities
    int16_t *tvr;   // [kMaxRows][kMaxTiles][hd/C]
    int32_t *mloc;  // [kMaxRows][kMaxTiles]
    int32_t *gsum;  // [kMaxRows][kMaxTiles]
    int32_t *gold;  // [kMaxRows][kMaxTiles]
    int32_t *tsum;  // [kMaxRows][tpc]
    uint32_t *qb;   // [kMaxRows][hd/2] query pairs as dp2a bytes
    uint8_t *ksat;  // [tpc*64] position holds a k >= 2048
    int32_t *vsat;  // [tpc] tile holds a v >= 2048; [tpc + r] = query row r holds -32768
};

static __host__ __device__ size_t attn_rows_layout(int tpc, int cl, size_t off[12]) {
    const size_t P = (size_t)tpc * kTile;
    size_t b = 0;
    off[0] = b; b = align16(b + P * kKvStride * 2);
    off[1] = b; b = align16(b + 2049 * 2);
    off[2] = b; b = align16(b + (size_t)kMaxRows * kMaxHd * 2);
    off[3] = b; b = align16(b + (size_t)kMaxRows * P * 2);
    off[4] = b; b = align16(b + (size_t)kMaxRows * kMaxTiles * (kMaxHd / cl) * 2);
    off[5] = b; b = align16(b + (size_t)kMaxRows * kMaxTiles * 4);
    off[6] = b; b = align16(b + (size_t)kMaxRows * kMaxTiles * 4);
    off[7] = b; b = align16(b + (size_t)kMaxRows * kMaxTiles * 4);
    off[8] = b; b = align16(b + (size_t)kMaxRows * tpc * 4);
    off[9] = b; b = align16(b + (size_t)kMaxRows * kMaxHd * 2);
    off[10] = b; b = align16(b + P);
    off[11] = b; b = align16(b + (size_t)(tpc + kMaxRows) * 4);
    return b;
}

size_t attn_rows_smem_bytes(int tpc, int cluster) {
    size_t off[12];
    return attn_rows_layout(tpc, cluster, off);
}

constexpr int kAttnRowsThreads = 256;

template <int C>
__global__ void __launch_bounds__(kAttnRowsThreads) k_attn_rows(const AttnArgs a) {
    extern __shared__ __align__(16) char raw[];
    cg::cluster_group cluster = cg::this_cluster();
    const int c = (int)cluster.block_rank();
    const int lh = blockIdx.x / C;
    const int hd = a.hd, vpr = hd >> 3, epc = hd / C;
    size_t off[12];
    attn_rows_layout(a.tpc_max, C, off);
    AttnRowsSmem m;
    m.qb = reinterpret_cast<uint32_t *>(raw + off[9]);
    m.ksat = reinterpret_cast<uint8_t *>(raw + off[10]);
    m.vsat = reinterpret_cast<int32_t *>(raw + off[11]);
    m.kv = reinterpret_cast<int16_t *>(raw + off[0]);
    m.ptab = reinterpret_cast<int16_t *>(raw + off[1]);
    m.q = reinterpret_cast<int16_t *>(raw + off[2]);
    m.sc = reinterpret_cast<int16_t *>(raw + off[3]);
    m.tvr = reinterpret_cast<int16_t *>(raw + off[4]);
    m.mloc = reinterpret_cast<int32_t *>(raw + off[5]);
    m.gsum = reinterpret_cast<int32_t *>(raw + off[6]);
    m.gold = reinterpret_cast<int32_t *>(raw + off[7]);
    m.tsum = reinterpret_cast<int32_t *>(raw + off[8]);
    const int P = a.tpc_max * kTile;  // row stride of sc

    for (int i = threadIdx.x; i < 2049; i += blockDim.x) m.ptab[i] = a.ptab[i];
    pdl_wait();
    pdl_trigger();
    const Step st = *a.step;
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

    for (int i = threadIdx.x; i < npos * vpr; i += blockDim.x) {
        const int pp = i / vpr, cc = (i - pp * vpr) << 3;
        cp_async16(m.kv + pp * kKvStride + cc, kb + (size_t)pp * hd + cc);
    }
    for (int i = threadIdx.x; i < R * vpr; i += blockDim.x) {
        const int r = i / vpr, v = i - r * vpr;
        reinterpret_cast<uint4 *>(m.q + r * kMaxHd)[v] =
            reinterpret_cast<const uint4 *>(a.q + (size_t)r * a.q_heads * hd + (size_t)lh * hd)[v];
    }
    for (int i = threadIdx.x; i < R * tpc; i += blockDim.x) m.tsum[i] = 0;
    for (int i = threadIdx.x; i < npos; i += blockDim.x) m.ksat[i] = 0;
    for (int i = threadIdx.x; i < tpc + kMaxRows; i += blockDim.x) m.vsat[i] = 0;
    cp_async_wait_all();
    __syncthreads();
    // clamp K in place (flagging positions with a k >= 2048); queries -> dp2a bytes
    for (int i = threadIdx.x; i < npos * vpr; i += blockDim.x) {
        const int pp = i / vpr, cc = (i - pp * vpr) << 3;
        uint4 *kp = reinterpret_cast<uint4 *>(m.kv + pp * kKvStride + cc);
        uint4 kv = *kp;
        if (clamp_k12(kv)) m.ksat[pp] = 1;
        *kp = kv;
    }
    for (int i = threadIdx.x; i < R * vpr; i += blockDim.x) {
        const int r = i / vpr, v = i - r * vpr;
        const uint4 qv = reinterpret_cast<const uint4 *>(m.q + r * kMaxHd)[v];
        if ((__vcmpeq2(qv.x, 0x80008000u) | __vcmpeq2(qv.y, 0x80008000u) | __vcmpeq2(qv.z, 0x80008000u) |
             __vcmpeq2(qv.w, 0x80008000u)) != 0)
            m.vsat[tpc + r] = 1;
        reinterpret_cast<uint4 *>(m.qb + r * (kMaxHd / 2))[v] =
            make_uint4(q_pair_bytes(qv.x), q_pair_bytes(qv.y), q_pair_bytes(qv.z), q_pair_bytes(qv.w));
    }
    __syncthreads();

    // ---- 1. scores of every (row, position) of the row's context -----------
    for (int i = threadIdx.x; i < R * npos; i += blockDim.x) {
        const int r = i / npos, pp = i - r * npos;
        if (pp >= npos_of(r)) continue;
        const int16_t *qg = a.q + (size_t)r * a.q_heads * hd + (size_t)lh * hd;
        int32_t tot = m.ksat[pp] || m.vsat[tpc + r]
                          ? qk_dot_exact(qg, kb + (size_t)pp * hd, hd)
                          : qk_dot_fast(reinterpret_cast<const uint4 *>(m.kv + pp * kKvStride),
                                        reinterpret_cast<const uint4 *>(m.qb + r * (kMaxHd / 2)), vpr);
        tot = sat32(rnd((int64_t)tot * a.qk_scale, 16));
        m.sc[r * P + pp] = (int16_t)sat16(rnd(tot, 8));
    }
    __syncthreads();  // K consumed: the buffer now receives V
    for (int i = threadIdx.x; i < npos * vpr; i += blockDim.x) {
        const int pp = i / vpr, cc = (i - pp * vpr) << 3;
        cp_async16(m.kv + pp * kKvStride + cc, vb + (size_t)pp * hd + cc);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
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
        if (pp >= npos_of(r)) {  // outside row r's context: probability 0 adds nothing to PV
            m.sc[r * P + pp] = 0;
            continue;
        }
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
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    __syncthreads();
    for (int i = threadIdx.x; i < npos * vpr; i += blockDim.x) {  // clamp V in place, flag tiles with v >= 2048
        const int pp = i / vpr, cc = (i - pp * vpr) << 3;
        uint4 *vp = reinterpret_cast<uint4 *>(m.kv + pp * kKvStride + cc);
        uint4 vv = *vp;
        if (clamp_k12(vv)) m.vsat[pp / kTile] = 1;
        *vp = vv;
    }
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
    __syncthreads();  // V clamped, tiles flagged, probabilities final
    // PV: one (tile, element pair) per item, its V words read once for every row
    for (int i = threadIdx.x; i < nown * (hd >> 1); i += blockDim.x) {
        const int tli = i / (hd >> 1), e = 2 * (i - tli * (hd >> 1));
        const int pb = tli * kTile, pe = min(pb + kTile, npos);
        int32_t acc[kMaxRows][2];
#pragma unroll
        for (int r = 0; r < kMaxRows; r++) acc[r][0] = acc[r][1] = 0;
        if (m.vsat[tli]) {
            for (int r = 0; r < R; r++) {
                const int n = max(0, min(pe, npos_of(r)) - pb);
                acc[r][0] = pv_exact(m.sc + r * P + pb, vb + (size_t)pb * hd + e, hd, n);
                acc[r][1] = pv_exact(m.sc + r * P + pb, vb + (size_t)pb * hd + e + 1, hd, n);
            }
        } else {
            for (int pp = pb; pp < pe; pp++) {
                const uint32_t w = *reinterpret_cast<const uint32_t *>(m.kv + pp * kKvStride + e);
                const int32_t v0 = lo16(w), v1 = hi16(w);
#pragma unroll
                for (int r = 0; r < kMaxRows; r++)
                    if (r < R) {
                        const int32_t pr = m.sc[r * P + pp];
                        acc[r][0] += pr * v0;
                        acc[r][1] += pr * v1;
                    }
            }
        }
#pragma unroll
        for (int r = 0; r < kMaxRows; r++) {
            if (r >= R || t_begin + tli >= ntiles_of(r)) continue;
#pragma unroll
            for (int h = 0; h < 2; h++) {
                const int32_t ts = sat32(rnd((int64_t)acc[r][h] * 1024, 16));
                const int16_t tv = (int16_t)sat16(rnd(ts, 8));
                *cluster.map_shared_rank(m.tvr + (r * kMaxTiles + t_begin + tli) * epc + (e + h) / C, (e + h) % C) = tv;
            }
        }
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

cudaError_t attn_rows_configure(int max_smem_bytes, int cluster) {
    if (cluster == kClusterWide) {
        cudaError_t e = cudaFuncSetAttribute(k_attn_rows<kClusterWide>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
        if (e != cudaSuccess) return e;
        return cudaFuncSetAttribute(k_attn_rows<kClusterWide>, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem_bytes);
    }
    return cudaFuncSetAttribute(k_attn_rows<kCluster>, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem_bytes);
}

cudaError_t launch_attn_rows(const AttnArgs &a, cudaStream_t s) {
    AttnArgs c = a;
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
    const void *fn = a.cluster == kClusterWide ? (const void *)k_attn_rows<kClusterWide> : (const void *)k_attn_rows<kCluster>;
    return cudaLaunchKernelExC(&cfg, fn, args);
}

cudaError_t attn_configure(int max_smem_bytes, int cluster) {
    if (cluster == kClusterWide) {
        cudaError_t e = cudaFuncSetAttribute(k_attn<kClusterWide>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
        if (e != cudaSuccess) return e;
        return cudaFuncSetAttribute(k_attn<kClusterWide>, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem_bytes);
    }
    return cudaFuncSetAttribute(k_attn<kCluster>, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem_bytes);
}

cudaError_t launch_attn(const AttnArgs &a, int rows, cudaStream_t s) {
    AttnArgs c = a;
    void *args[] = {&c};
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.cluster * a.q_heads, rows);
    cfg.blockDim = dim3(kAttnThreads);
    cfg.dynamicSmemBytes = attn_smem_bytes(a.tpc_max, a.hd, a.cluster);
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
    const void *fn = a.cluster == kClusterWide ? (const void *)k_attn<kClusterWide> : (const void *)k_attn<kCluster>;
    return cudaLaunchKernelExC(&cfg, fn, args);
}

}  // namespace llmx
