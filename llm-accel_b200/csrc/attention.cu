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
// One thread-block cluster of kCluster CTAs handles one (row, query head).
// CTA c owns the contiguous tiles [c*tpc, (c+1)*tpc):
//   1. K and V rows of its tiles land in shared memory (cp.async, issued
//      together); QK scores of its positions and its tile maxima;
//   2. cluster barrier; running maxima from all owners' tile maxima (DSMEM);
//      Q2.14 probabilities, tile sums, rescale factors and the raw-payload PV
//      tile values of its tiles;
//   3. cluster barrier; the (sum, acc) recurrence in tile order, each CTA
//      finalising hd/kCluster output elements from the owners' tile values;
//   4. cluster barrier, so no CTA leaves while its shared memory is read.
// All waits are hardware cluster barriers: no flags, no spin loops, and no
// global scratch memory.
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

struct AttnSmem {   // carved out of dynamic shared memory
    int16_t *k, *v; // [tpc*64][kKvStride] raw Q8.8 rows of the owned tiles
    int16_t *q;     // [hd]
    int16_t *sc;    // [tpc*64] scores, then Q2.14 probabilities
    int16_t *tval;  // [tpc][hd] owned PV tile values (Q8.8)
    int32_t *tmax;  // [tpc] owned tile maxima
    int32_t *tsum;  // [tpc] owned tile sums (Q16.16)
    int32_t *told;  // [tpc] owned rescale factors (Q2.14)
    int32_t *mall;  // [kCluster*tpc] running max after every tile
    int32_t *gsum;  // [kCluster*tpc] gathered tile sums
    int32_t *gold;  // [kCluster*tpc] gathered rescale factors
};

static __host__ __device__ size_t align16(size_t b) { return (b + 15) & ~size_t(15); }

static __host__ __device__ size_t attn_layout(int tpc, int hd, size_t off[10]) {
    const size_t rows = (size_t)tpc * kTile;
    size_t b = 0;
    off[0] = b; b = align16(b + rows * kKvStride * 2);           // k
    off[1] = b; b = align16(b + rows * kKvStride * 2);           // v
    off[2] = b; b = align16(b + (size_t)kMaxHd * 2);             // q
    off[3] = b; b = align16(b + rows * 2);                       // sc
    off[4] = b; b = align16(b + (size_t)tpc * hd * 2);           // tval
    off[5] = b; b = align16(b + (size_t)tpc * 4);                // tmax
    off[6] = b; b = align16(b + (size_t)tpc * 4);                // tsum
    off[7] = b; b = align16(b + (size_t)tpc * 4);                // told
    off[8] = b; b = align16(b + (size_t)kCluster * tpc * 4);     // mall
    off[9] = b; b = align16(b + (size_t)kCluster * tpc * 4 * 2); // gsum, gold
    return b;
}

size_t attn_smem_bytes(int tpc, int hd) {
    size_t off[10];
    return attn_layout(tpc, hd, off);
}

__global__ void __launch_bounds__(kAttnThreads) k_attn(const AttnArgs a) {
    extern __shared__ __align__(16) char raw[];
    cg::cluster_group cluster = cg::this_cluster();
    const int c = (int)cluster.block_rank();
    const int lh = blockIdx.x / kCluster;  // local query head
    const int r = blockIdx.y;
    const int hd = a.hd, vpr = hd >> 3;
    size_t off[10];
    attn_layout(a.tpc_max, hd, off);
    AttnSmem m;
    m.k = reinterpret_cast<int16_t *>(raw + off[0]);
    m.v = reinterpret_cast<int16_t *>(raw + off[1]);
    m.q = reinterpret_cast<int16_t *>(raw + off[2]);
    m.sc = reinterpret_cast<int16_t *>(raw + off[3]);
    m.tval = reinterpret_cast<int16_t *>(raw + off[4]);
    m.tmax = reinterpret_cast<int32_t *>(raw + off[5]);
    m.tsum = reinterpret_cast<int32_t *>(raw + off[6]);
    m.told = reinterpret_cast<int32_t *>(raw + off[7]);
    m.mall = reinterpret_cast<int32_t *>(raw + off[8]);
    m.gsum = reinterpret_cast<int32_t *>(raw + off[9]);
    m.gold = m.gsum + kCluster * a.tpc_max;

    pdl_wait();
    pdl_trigger();
    const Step st = *a.step;
    // every CTA of the cluster reaches every barrier, also when it owns nothing
    const bool row_ok = r < st.rows;
    const int ctx = st.position + r + 1;
    const int ntiles = row_ok ? (ctx + kTile - 1) / kTile : 0;
    const int tpc = max(1, (ntiles + kCluster - 1) / kCluster);
    const int t_begin = min(c * tpc, ntiles), t_end = min(t_begin + tpc, ntiles);
    const int nown = t_end - t_begin;
    const int p_begin = t_begin * kTile;
    const int npos = nown > 0 ? min(t_end * kTile, ctx) - p_begin : 0;
    const int kvh = (a.first_head + lh) / a.gqa;

    if (npos > 0) {
        const int16_t *kb = a.kc + ((size_t)kvh * a.max_seq + p_begin) * hd;
        const int16_t *vb = a.vc + ((size_t)kvh * a.max_seq + p_begin) * hd;
        for (int i = threadIdx.x; i < npos * vpr; i += blockDim.x) {
            const int pp = i / vpr, cc = (i - pp * vpr) << 3;
            cp_async16(m.k + pp * kKvStride + cc, kb + (size_t)pp * hd + cc);
            cp_async16(m.v + pp * kKvStride + cc, vb + (size_t)pp * hd + cc);
        }
        const uint4 *qsrc = reinterpret_cast<const uint4 *>(a.q + (size_t)r * a.q_heads * hd + (size_t)lh * hd);
        for (int i = threadIdx.x; i < vpr; i += blockDim.x) reinterpret_cast<uint4 *>(m.q)[i] = qsrc[i];
        for (int i = threadIdx.x; i < nown; i += blockDim.x) {
            m.tmax[i] = -32768;
            m.tsum[i] = 0;
        }
        cp_async_wait_all();
    }
    __syncthreads();

    // ---- 1. scores and owned tile maxima ---------------------------------
    for (int pp = threadIdx.x; pp < npos; pp += blockDim.x) {
        const uint4 *qv = reinterpret_cast<const uint4 *>(m.q);
        const uint4 *kv = reinterpret_cast<const uint4 *>(m.k + pp * kKvStride);
        int32_t b0 = 0, b1 = 0, b2 = 0, b3 = 0;  // banks k mod 4, saturating, in k order
        for (int e8 = 0; e8 < vpr; e8++) {
            const uint4 q = qv[e8], k = kv[e8];
            b0 = add_sat(b0, qk_prod(lo16(q.x), q412(lo16(k.x))));
            b1 = add_sat(b1, qk_prod(hi16(q.x), q412(hi16(k.x))));
            b2 = add_sat(b2, qk_prod(lo16(q.y), q412(lo16(k.y))));
            b3 = add_sat(b3, qk_prod(hi16(q.y), q412(hi16(k.y))));
            b0 = add_sat(b0, qk_prod(lo16(q.z), q412(lo16(k.z))));
            b1 = add_sat(b1, qk_prod(hi16(q.z), q412(hi16(k.z))));
            b2 = add_sat(b2, qk_prod(lo16(q.w), q412(lo16(k.w))));
            b3 = add_sat(b3, qk_prod(hi16(q.w), q412(hi16(k.w))));
        }
        int32_t tot = sat32((int64_t)b0 + b1 + b2 + b3);
        tot = sat32(rnd((int64_t)tot * a.qk_scale, 16));  // x accum(fm(1/sqrt(d)))
        const int32_t sc = sat16(rnd(tot, 8));
        m.sc[pp] = (int16_t)sc;
        atomicMax(m.tmax + pp / kTile, sc);
    }
    cluster.sync();

    // ---- 2. running maxima, probabilities, tile sums, rescale, PV --------
    if (threadIdx.x == 0 && nown > 0) {
        int32_t run = -32768;  // m_{-1} = fm(-128)
        for (int t = 0; t < t_end; t++) {
            const int owner = t / tpc;
            run = max(run, *cluster.map_shared_rank(m.tmax + (t - owner * tpc), owner));
            m.mall[t] = run;
        }
    }
    __syncthreads();
    for (int i = threadIdx.x; i < nown; i += blockDim.x) {
        const int t = t_begin + i;
        const int32_t mprev = t > 0 ? m.mall[t - 1] : -32768;
        int32_t d = sat16(mprev - m.mall[t]);
        d = d < -2048 ? -2048 : d;
        m.told[i] = __ldg(a.ptab + d + 2048);
    }
    for (int pp = threadIdx.x; pp < npos; pp += blockDim.x) {
        int32_t d = sat16((int32_t)m.sc[pp] - m.mall[t_begin + pp / kTile]);
        d = d < -2048 ? -2048 : (d > 0 ? 0 : d);
        const int32_t pr = __ldg(a.ptab + d + 2048);
        m.sc[pp] = (int16_t)pr;
        atomicAdd(m.tsum + pp / kTile, pr * 4);  // Q2.14 -> Q16.16; <= 64 * 2^16, never saturates
    }
    __syncthreads();
    // raw payload p (read as Q8.8) x V (Q4.12, saturated), rounded per product,
    // four banks in position order (|p*v| <= 2^29: banks never saturate),
    // x accum(fm(1/64)), -> fm
    for (int i = threadIdx.x; i < nown * hd; i += blockDim.x) {
        const int tli = i / hd, e = i - tli * hd;
        const int pb = tli * kTile, pe = min(pb + kTile, npos);
        int32_t b0 = 0, b1 = 0, b2 = 0, b3 = 0;
        int pp = pb;
        for (; pp + 3 < pe; pp += 4) {
            b0 += qk_prod(m.sc[pp], q412(m.v[pp * kKvStride + e]));
            b1 += qk_prod(m.sc[pp + 1], q412(m.v[(pp + 1) * kKvStride + e]));
            b2 += qk_prod(m.sc[pp + 2], q412(m.v[(pp + 2) * kKvStride + e]));
            b3 += qk_prod(m.sc[pp + 3], q412(m.v[(pp + 3) * kKvStride + e]));
        }
        if (pp < pe) b0 += qk_prod(m.sc[pp], q412(m.v[pp * kKvStride + e]));
        if (pp + 1 < pe) b1 += qk_prod(m.sc[pp + 1], q412(m.v[(pp + 1) * kKvStride + e]));
        if (pp + 2 < pe) b2 += qk_prod(m.sc[pp + 2], q412(m.v[(pp + 2) * kKvStride + e]));
        int32_t ts = sat32((int64_t)b0 + b1 + b2 + b3);
        ts = sat32(rnd((int64_t)ts * 1024, 16));
        m.tval[tli * hd + e] = (int16_t)sat16(rnd(ts, 8));
    }
    cluster.sync();

    // ---- 3. in-order Q16.16 recurrence ------------------------------------
    for (int i = threadIdx.x; i < ntiles; i += blockDim.x) {
        const int owner = i / tpc;
        m.gsum[i] = *cluster.map_shared_rank(m.tsum + (i - owner * tpc), owner);
        m.gold[i] = *cluster.map_shared_rank(m.told + (i - owner * tpc), owner);
    }
    __syncthreads();
    for (int e = c + kCluster * (int)threadIdx.x; ntiles > 0 && e < hd; e += kCluster * blockDim.x) {
        int32_t sum = 0, acc = 0;
        for (int u0 = 0; u0 < ntiles; u0 += 8) {
            int32_t tv[8];
#pragma unroll
            for (int j = 0; j < 8; j++) {  // fetch 8 tiles' values before using them
                const int u = u0 + j, owner = u / tpc;
                tv[j] = u < ntiles ? *cluster.map_shared_rank(m.tval + (u - owner * tpc) * hd + e, owner) : 0;
            }
#pragma unroll
            for (int j = 0; j < 8; j++) {
                const int u = u0 + j;
                if (u < ntiles) {
                    const int64_t o = (int64_t)m.gold[u] * 4;  // Q2.14 -> Q16.16
                    sum = sat32(rnd((int64_t)sum * o, 16) + m.gsum[u]);
                    acc = sat32(rnd((int64_t)acc * o, 16));
                    acc = sat32((int64_t)acc + (int64_t)tv[j] * 256);
                }
            }
        }
        const int64_t safe = sum < 16 ? 16 : sum;
        const int64_t quot = ((int64_t)1 << 32) / safe;  // accum(1) / safe: 16 fraction bits, truncated
        const int64_t inv = sat16(rnd(quot, 8));
        a.out[(size_t)r * a.q_heads * hd + (size_t)lh * hd + e] = (int16_t)sat16(rnd(acc * inv * 256, 24));
    }
    cluster.sync();
}

cudaError_t attn_configure(int max_smem_bytes) {
    return cudaFuncSetAttribute(k_attn, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem_bytes);
}

cudaError_t launch_attn(const AttnArgs &a, int rows, cudaStream_t s) {
    AttnArgs c = a;
    void *args[] = {&c};
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(kCluster * a.q_heads, rows);
    cfg.blockDim = dim3(kAttnThreads);
    cfg.dynamicSmemBytes = attn_smem_bytes(a.tpc_max, a.hd);
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = kCluster;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    return cudaLaunchKernelExC(&cfg, (const void *)k_attn, args);
}

}  // namespace llmx
