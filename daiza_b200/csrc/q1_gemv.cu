// q1_gemv.cu -- Q1_0 projection GEMV for a few tokens on the integer tensor
// cores (warp-level mma.sync, see "Why mma.sync" below).
//
// Reference: Daiza-engine/src/model/weights.rs:831 (matvec_multi_into_slice: up
// to 8 Q1_0 matrices sharing one input row), weights.rs:334
// (matvec_add_into_slice: y += W x) with the row kernel tensor/quant.rs:267-328
// (dot_q1_0_row_avx2) and its multi-token twin (weights.rs verify4t path).
// Q1_0 row layout: cols/128 blocks of 18 bytes -- the group scale as IEEE
// binary16 (little endian), then 16 sign bytes whose bit b of byte j is weight
// 8j + b (1 -> +scale, 0 -> -scale).
//
// With s_i = +-1 the signs of a group, sum_i s_i x_i = 2 sum_{bit_i = 1} x_i - sum_i x_i,
// and both sums are exact in integers once x is in fixed point:
//   1. q1_prep (one warp per (token, group of 128 inputs)): x ~= s_tg q with
//      |q| <= QMAX and s_tg = max|x over the group| / QMAX; q = 65536 d2 +
//      256 d1 + d0 with signed 8-bit digits.  Column n = 3t + p of the MMA's
//      B operand is digit plane p of token t (NB blocks of 8 columns, unused
//      columns zero); prep writes the B fragments of mma.m16n8k32 in register
//      order, per group and K step, plus per column the factor 2 * 256^p * s_tg
//      and (plane 0 only) the term s_tg * sum q.
//   2. q1_gemv (a programmatic dependent of 1): the work is a list of items
//      (128-row block, 8 groups); each cluster takes a contiguous range of row
//      blocks and each CTA of it a range of every block's items.  A loader
//      thread brings each item's 128 x 144 weight bytes (one 2-D TMA box of
//      the Q1_0 rows) and its 8 groups of B fragments into a two-slot ring.  Warp w of 8 takes rows 16w .. 16w+15: per group, lane
//      (g, q) reads sign word q of rows g and g+8 and turns it into A fragments
//      with (word >> s) & 0x01010101 -- bits s, s+8, s+16, s+24 as 0/1 bytes --
//      so K step s of the group uses bits s and s+4 of every word, and the B
//      fragments follow the same order.  mma.sync.m16n8k32 (s8 x s8 -> s32)
//      sums the set bits' digits exactly over the group; each int32 column
//      value then enters an f32 sum per (row, column) as
//      scale * (factor * a - term).  When a block is complete the 3 plane
//      columns of each token are added into y.  When there are fewer row
//      blocks than CTA slots, a block's units are split over a cluster of 2 or
//      4 CTAs; each stores its row sums into rank 0's shared memory (distributed
//      shared memory) and rank 0 adds them in rank order, so results do not
//      depend on timing.
// Why mma.sync: a tcgen05.mma kind::i8 with M = 128 and K = 32 takes about 58
// cycles per SM at any N up to 64 (143 at N = 256), so with N = 3T <= 24 it
// processes 128 x 32 weights per ~58 cycles -- about 70 weights per cycle per
// SM, under half of the HBM rate.  The register-operand m16n8k32 runs at about
// 0.4 per cycle per SM (512 weights each, ~200 weights per cycle) and needs no
// staging of the expanded signs in shared or tensor memory.
// The only rounding beyond f32 accumulation is the input quantisation (~1e-7 of
// the group's max|x| per element).  Roofline: HBM -- the Q1_0 bytes (1.125 bits
// per weight) are read once.
#include <cuda.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <cstddef>

#include "dz_internal.h"
#include "tc_common.cuh"

namespace dz {

namespace q1 {
constexpr int ROWS = 128;                    // rows per item
constexpr int UNIT = 8;                      // groups per item
constexpr int UNIT_BYTES = UNIT * 18;        // 144 bytes of each row per item
constexpr int WBYTES = ROWS * UNIT_BYTES;    // 18432: one item's weights
constexpr int NS = 2;                        // item slots in shared memory
constexpr int CWARPS = 8;                    // compute warps (16 rows each)
constexpr int THREADS = 32 * (CWARPS + 1);   // + one loader warp
constexpr int CTAS_PER_SM = 2;
constexpr int QMAX = 8355000;                // |q| bound: three signed 8-bit digits reach +-8,355,711
constexpr int PLANES = 3;
constexpr int PREP_WARPS = 8;
constexpr int MAX_BLOCKS = 4096;             // row blocks per call
}  // namespace q1

// column blocks of 8 (3T columns) and the prepared bytes of one group:
// B fragments [NB][32 lanes][4 K steps][2 words], then per block and lane quad q the
// column pair's (factor, factor, term, term) as f32 [NB][4][4]
__host__ __device__ inline int q1_nb(int T) { return (3 * T + 7) / 8; }
__host__ __device__ inline int q1_group_bytes(int T) { return q1_nb(T) * (4 * 256 + 64); }

constexpr int Q1_MAX_KS = 4;                 // CTAs per cluster: 1, 2 or 4

size_t q1_smem_bytes(int cols, int T) {
    (void)cols;
    const size_t slot = (size_t)q1::WBYTES + (size_t)q1::UNIT * q1_group_bytes(T);
    return 128 + q1::NS * slot + (size_t)q1::ROWS * 25 * 4 + (size_t)Q1_MAX_KS * q1::ROWS * T * 4 + 64;
}
int q1_max_blocks() { return q1::MAX_BLOCKS; }

struct Q1Desc {
    CUtensorMap map[Q1_MAX_MATS];   // the Q1_0 rows of each matrix as a [rows][rowbytes] byte tensor
    float* y[Q1_MAX_MATS];
    int rows[Q1_MAX_MATS];
    int blk0[Q1_MAX_MATS + 1];      // first 128-row block of each matrix
    int n_mats, cols, T, accumulate;
    int units;                      // items per row block (groups / 8)
    int ks;                         // CTAs per cluster sharing each row block's units
};

// ---------------------------------------------------------------------------
// 1. input preparation: grid (ceil(groups / 8), T), one warp per (token, group)
// ---------------------------------------------------------------------------
// Lane l holds inputs 4l .. 4l+3 of the group.  B fragment word b0 of lane
// (n, q) for K step s is the digits of column n at inputs 32q + s + 8b
// (b = 0..3), word b1 the same at 32q + s + 4 + 8b.
__global__ void __launch_bounds__(32 * q1::PREP_WARPS) q1_prep_kernel(const float* __restrict__ x, int cols, int T,
                                                                      unsigned char* __restrict__ prep) {
    using namespace q1;
    // the GEMV may start (and stream its weights) now; x and the scratch it reads are
    // the predecessor's, so wait for that grid before touching them
    asm volatile("griddepcontrol.launch_dependents;");
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int t = blockIdx.y, lane = threadIdx.x & 31;
    const int groups = cols / 128;
    const int g = blockIdx.x * PREP_WARPS + (threadIdx.x >> 5);
    if (g >= groups) return;
    const int NB = q1_nb(T);
    unsigned char* gp = prep + (size_t)g * q1_group_bytes(T);
    const float4 v4 = reinterpret_cast<const float4*>(x + (size_t)t * cols + (size_t)g * 128)[lane];
    const float v[4] = {v4.x, v4.y, v4.z, v4.w};
    float mx = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
    mx = warp_max(mx);
    const float inv = mx > 0.0f ? (float)QMAX / mx : 0.0f;
    int dg[PLANES][4];
    int s4 = 0;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        int q = __float2int_rn(v[e] * inv);
        q = max(-QMAX, min(QMAX, q));
        s4 += q;
#pragma unroll
        for (int p = 0; p < PLANES; ++p) {
            const int dgt = ((q + 128) & 255) - 128;   // digit in [-128, 127]
            dg[p][e] = dgt & 0xFF;
            q = (q - dgt) >> 8;                        // exact division
        }
    }
    const int S = __reduce_add_sync(0xffffffffu, s4);   // |S| <= 128 QMAX < 2^31
    const float sx = mx > 0.0f ? mx / (float)QMAX : 0.0f;
    // input i = 4 lane + e is K position (4 q' + b) of K step s' with
    // q' = i / 32, s' = i % 8 (bits s', s'+8, ... of word q'), b = (i % 32) / 8
    // -- so lane l = 8 q' + 2 b + (s' / 4) holds it at e = s' % 4 (word b0 if s' < 4, else b1)
    uint32_t* frag = reinterpret_cast<uint32_t*>(gp);
#pragma unroll
    for (int p = 0; p < PLANES; ++p) {
        const int n = 3 * t + p, nb = n >> 3, ng = n & 7;
        // word (s, half) of fragment lane (ng, q') gathers byte e = s of lanes 8q' + 2b + half, b = 0..3
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const uint32_t mine = (uint32_t)dg[p][e];
            const int src_q = lane >> 3, src_b = (lane >> 1) & 3, half = lane & 1;
            // lanes with the same (q', half) build one word: OR of their bytes at position b
            uint32_t w = mine << (8 * src_b);
            w |= __shfl_xor_sync(0xffffffffu, w, 2);
            w |= __shfl_xor_sync(0xffffffffu, w, 4);
            if (src_b == 0)
                frag[(((size_t)nb * 32 + ng * 4 + src_q) * 4 + e) * 2 + half] = w;
        }
    }
    // unused columns of the last block: zero fragments and factors (written by token 0)
    if (t == 0)
        for (int n = 3 * T; n < 8 * NB; ++n) {
            const int nb = n >> 3, ng = n & 7;
            if (lane < 8) {
                const int e = lane >> 1, half = lane & 1;
#pragma unroll
                for (int qq = 0; qq < 4; ++qq) frag[(((size_t)nb * 32 + ng * 4 + qq) * 4 + e) * 2 + half] = 0u;
            }
        }
    // column n: block n / 8, quad (n % 8) / 2, slot n % 2
    float* ft = reinterpret_cast<float*>(gp + (size_t)NB * 4 * 256);
    auto ft_at = [&](int n) { return ft + ((n >> 3) * 4 + ((n & 7) >> 1)) * 4 + (n & 1); };
    if (lane < PLANES) {
        const int n = 3 * t + lane;
        ft_at(n)[0] = 2.0f * (float)(1 << (8 * lane)) * sx;
        ft_at(n)[2] = lane == 0 ? sx * (float)S : 0.0f;
    }
    if (t == 0 && lane < 8 * NB - 3 * T) {
        ft_at(3 * T + lane)[0] = 0.0f;
        ft_at(3 * T + lane)[2] = 0.0f;
    }
}

// ---------------------------------------------------------------------------
// 2. the GEMV
// ---------------------------------------------------------------------------
// Bounded wait without a suspend-time hint: the hand-offs here are short and
// frequent, so a waiting warp should resume as soon as the phase completes.
template <bool CLUSTER = false>
__device__ __forceinline__ bool q1_wait(uint64_t* bar, uint32_t parity, int* err, bool& ok) {
    if (!ok) return false;
    uint32_t done;
    const uint64_t t0 = global_ns();
    for (uint32_t i = 0;; ++i) {
        if (CLUSTER)
            asm volatile(
                "{\n\t.reg .pred p;\n\t"
                "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
                "selp.u32 %0, 1, 0, p;\n\t}"
                : "=r"(done) : "r"(smem_u32(bar)), "r"(parity) : "memory");
        else
            asm volatile(
                "{\n\t.reg .pred p;\n\t"
                "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
                "selp.u32 %0, 1, 0, p;\n\t}"
                : "=r"(done) : "r"(smem_u32(bar)), "r"(parity) : "memory");
        if (done) return true;
        if ((i & 15u) == 15u && global_ns() - t0 > MBAR_WAIT_LIMIT_NS) break;
    }
    atomicExch(err, DEVERR_MBAR_TIMEOUT);
    ok = false;
    return false;
}

__device__ __forceinline__ void mma_s8(int* d, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                       uint32_t b1) {
    asm volatile("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                 : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
                 : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// 32-bit word at a 2-byte aligned shared-memory address
__device__ __forceinline__ uint32_t lds_u32_a2(const unsigned char* p) {
    const uint32_t lo = *reinterpret_cast<const unsigned short*>(p);
    const uint32_t hi = *reinterpret_cast<const unsigned short*>(p + 2);
    return lo | (hi << 16);
}

// float(d) for |d| < 2^22 with one integer add and one float add (the
// conversion instruction has a quarter of the throughput): 0x4B400000 is
// 1.5 * 2^23, whose bit pattern plus d is exactly 1.5 * 2^23 + d
__device__ __forceinline__ float i2f_small(int d) { return __int_as_float(0x4B400000 + d) - 12582912.0f; }

// shared-memory address of the same variable in CTA `rank` of the cluster
__device__ __forceinline__ uint32_t cluster_addr(const void* p, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
    return r;
}
__device__ __forceinline__ void st_cluster_f32(uint32_t addr, float v) {
    asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}
__device__ __forceinline__ void arrive_cluster(uint32_t bar_addr) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar_addr) : "memory");
}
__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

// Work split: the row blocks are cut into equal contiguous ranges, one per
// cluster of KS CTAs; CTA rank r of a cluster takes units
// [r U / KS, (r+1) U / KS) of every block of its range.  Per block, every CTA
// of the cluster stores its row sums into rank 0's reduction buffer and rank 0
// adds them in rank order.
template <int NB>
__global__ void __launch_bounds__(q1::THREADS, q1::CTAS_PER_SM) q1_gemv_kernel(const __grid_constant__ Q1Desc d,
                                                                                const unsigned char* __restrict__ prep,
                                                                                int* err) {
    using namespace q1;
    constexpr int GB = NB * (4 * 256 + 64);     // prepared bytes per group
    constexpr int XBYTES = UNIT * GB;
    constexpr int SLOT = WBYTES + XBYTES;       // multiple of 128
    constexpr int NCOL = 8 * NB;
    constexpr int NT = CWARPS * 32;
    extern __shared__ unsigned char smem_raw[];
    unsigned char* smem = smem_raw + ((128 - (smem_u32(smem_raw) & 127)) & 127);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int U = d.units, T = d.T, KS = d.ks;
    const int clus = blockIdx.x / KS;
    const uint32_t rank = KS > 1 ? cluster_rank() : 0u;
    const int nclus = gridDim.x / KS, nblk = d.blk0[d.n_mats];
    const int b_begin = clus * nblk / nclus, b_end = (clus + 1) * nblk / nclus;
    const int u0 = (int)rank * U / KS, nu = ((int)rank + 1) * U / KS - u0;
    const int n_it = (b_end - b_begin) * nu;
    float* stage = reinterpret_cast<float*>(smem + NS * SLOT);          // [128][25] column sums of a block
    float* red = stage + ROWS * 25;                                     // [KS][128][T] row sums (rank 0)
    uint64_t* bars = reinterpret_cast<uint64_t*>(red + KS * ROWS * T + ((KS * ROWS * T) & 1));
    uint64_t* full = bars;                      // [NS] item landed
    uint64_t* empty = full + NS;                // [NS] item read by the compute warps
    uint64_t* red_full = empty + NS;            // rank 0: the other ranks stored their sums
    uint64_t* red_empty = red_full + 1;         // rank > 0: rank 0 has read the buffer

    auto item_of = [&](int k, int& m, int& r0, int& u) {
        const int b = b_begin + k / nu;
        u = u0 + k % nu;
        m = 0;
        while (b >= d.blk0[m + 1]) ++m;
        r0 = (b - d.blk0[m]) * ROWS;
    };
    const int pre = min(NS, n_it);
    if (warp == CWARPS && lane == 0) {
        for (int s = 0; s < NS; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], CWARPS);
        }
        mbar_init(red_full, CWARPS * (KS - 1) > 0 ? CWARPS * (KS - 1) : 1);
        mbar_init(red_empty, CWARPS);
        fence_mbar_init();
        // the weights do not depend on the preceding kernel: start them before anything else
        for (int k = 0; k < pre; ++k) {
            int m, r0, u;
            item_of(k, m, r0, u);
            mbar_arrive_expect_tx(&full[k], SLOT);
            tc::tma_load_2d(smem + k * SLOT, &d.map[m], u * UNIT_BYTES, r0, &full[k]);
        }
    }
    // barrier initialisation visible to the whole cluster before any remote arrive:
    // every thread arrives now and waits only before its first remote access
    if (KS > 1) asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
    __syncthreads();
    bool ok = true;

    if (warp == CWARPS) {
        // ---------------- loads (one thread) ----------------
        if (lane == 0) {
            asm volatile("griddepcontrol.wait;" ::: "memory");
            for (int k = 0; k < pre; ++k) {
                int m, r0, u;
                item_of(k, m, r0, u);
                bulk_g2s(smem + k * SLOT + WBYTES, prep + (size_t)u * XBYTES, XBYTES, &full[k]);
            }
            int k = pre;
            for (; k < n_it; ++k) {
                const int s = k % NS;
                if (!q1_wait(&empty[s], ((k / NS) - 1) & 1, err, ok)) break;
                int m, r0, u;
                item_of(k, m, r0, u);
                mbar_arrive_expect_tx(&full[s], SLOT);
                tc::tma_load_2d(smem + s * SLOT, &d.map[m], u * UNIT_BYTES, r0, &full[s]);
                bulk_g2s(smem + s * SLOT + WBYTES, prep + (size_t)u * XBYTES, XBYTES, &full[s]);
            }
            // copies still in flight when a wait gave up land before the CTA exits
            if (!ok)
                for (int j = max(0, k - NS); j < k; ++j) mbar_wait(&full[j % NS], (j / NS) & 1, err);
        }
        __syncwarp();
        if (KS > 1) asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
    } else {
        // ---------------- compute: warp w owns rows 16w .. 16w+15 of each item ----------------
        asm volatile("griddepcontrol.wait;" ::: "memory");
        const int g = lane >> 2, q = lane & 3;
        const int rA = 16 * warp + g, rB = rA + 8;
        float acc[NB][4];
#pragma unroll
        for (int nb = 0; nb < NB; ++nb)
#pragma unroll
            for (int i = 0; i < 4; ++i) acc[nb][i] = 0.0f;

        // a block's sums are complete: rank 0 of the cluster writes y
        auto flush = [&](int k, int blk_idx) {
#pragma unroll
            for (int nb = 0; nb < NB; ++nb) {
                stage[rA * 25 + nb * 8 + 2 * q] = acc[nb][0];
                stage[rA * 25 + nb * 8 + 2 * q + 1] = acc[nb][1];
                stage[rB * 25 + nb * 8 + 2 * q] = acc[nb][2];
                stage[rB * 25 + nb * 8 + 2 * q + 1] = acc[nb][3];
#pragma unroll
                for (int i = 0; i < 4; ++i) acc[nb][i] = 0.0f;
            }
            tc::named_bar_sync(1, NT);
            int m, r0, u;
            item_of(k, m, r0, u);
            const int rows = d.rows[m];
            const int nr = min(ROWS, rows - r0);
            float* yb = d.y[m] + r0;
            const int r = tid;                                   // threads 0..127: one row each
            float v[8];
#pragma unroll
            for (int t = 0; t < 8; ++t) v[t] = 0.0f;
            if (r < ROWS)
#pragma unroll
                for (int t = 0; t < 8; ++t)
                    if (3 * t + 2 < NCOL && t < T)
                        v[t] = stage[r * 25 + 3 * t] + stage[r * 25 + 3 * t + 1] + stage[r * 25 + 3 * t + 2];
            if (KS == 1) {
                if (r < nr)
#pragma unroll
                    for (int t = 0; t < 8; ++t)
                        if (t < T) {
                            float* yp = yb + (size_t)t * rows + r;
                            *yp = d.accumulate ? *yp + v[t] : v[t];
                        }
            } else if (rank != 0) {
                if (blk_idx == 0) asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
                // the buffer is free once rank 0 has read the previous block
                if (blk_idx > 0) ok = __all_sync(0xffffffffu, q1_wait<true>(red_empty, (blk_idx - 1) & 1, err, ok));
                if (r < ROWS) {
                    const uint32_t dst = cluster_addr(red + ((size_t)rank * ROWS + r) * T, 0);
#pragma unroll
                    for (int t = 0; t < 8; ++t)
                        if (t < T) st_cluster_f32(dst + 4 * t, v[t]);
                }
                // one release per warp covers the warp's stores (ordered by the warp barrier)
                __syncwarp();
                if (lane == 0) arrive_cluster(cluster_addr(red_full, 0));
            } else {
                if (blk_idx == 0) asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
                ok = __all_sync(0xffffffffu, q1_wait<true>(red_full, blk_idx & 1, err, ok));
                if (r < ROWS) {
                    float sum[8];
#pragma unroll
                    for (int t = 0; t < 8; ++t) sum[t] = v[t];
                    for (int rr = 1; rr < KS; ++rr) {
                        const float* pr = red + ((size_t)rr * ROWS + r) * T;
#pragma unroll
                        for (int t = 0; t < 8; ++t)
                            if (t < T) sum[t] += pr[t];
                    }
                    if (r < nr)
#pragma unroll
                        for (int t = 0; t < 8; ++t)
                            if (t < T) {
                                float* yp = yb + (size_t)t * rows + r;
                                *yp = d.accumulate ? *yp + sum[t] : sum[t];
                            }
                }
                // the other ranks may overwrite their parts now (after the last block
                // nothing touches their shared memory any more, so they may exit)
                __syncwarp();
                if (blk_idx < (b_end - b_begin) - 1 && lane == 0)
                    for (int rr = 1; rr < KS; ++rr) arrive_cluster(cluster_addr(red_empty, (uint32_t)rr));
            }
            tc::named_bar_sync(1, NT);                           // stage free for the next block
        };

        for (int k = 0; k < n_it; ++k) {
            const int s = k % NS;
            ok = __all_sync(0xffffffffu, q1_wait(&full[s], (k / NS) & 1, err, ok));
            const unsigned char* wA = smem + s * SLOT + rA * UNIT_BYTES;
            const unsigned char* wB = smem + s * SLOT + rB * UNIT_BYTES;
            const unsigned char* xp = smem + s * SLOT + WBYTES;
#pragma unroll
            for (int j = 0; j < UNIT; ++j) {
                // row scales (binary16 at byte 18j) and sign word q (bytes 18j + 2 + 4q:
                // 4-byte aligned for odd j)
                const float scA = __half2float(__ushort_as_half(*reinterpret_cast<const unsigned short*>(wA + 18 * j)));
                const float scB = __half2float(__ushort_as_half(*reinterpret_cast<const unsigned short*>(wB + 18 * j)));
                uint32_t swA, swB;
                if (j % 2 == 1) {
                    swA = *reinterpret_cast<const uint32_t*>(wA + 18 * j + 2 + 4 * q);
                    swB = *reinterpret_cast<const uint32_t*>(wB + 18 * j + 2 + 4 * q);
                } else {
                    swA = lds_u32_a2(wA + 18 * j + 2 + 4 * q);
                    swB = lds_u32_a2(wB + 18 * j + 2 + 4 * q);
                }
                const unsigned char* gp = xp + j * GB;
                int dacc[NB][4];
#pragma unroll
                for (int nb = 0; nb < NB; ++nb) {
                    // this lane's B fragments of the 4 K steps
                    const uint4 f01 = reinterpret_cast<const uint4*>(gp)[(nb * 32 + lane) * 2];
                    const uint4 f23 = reinterpret_cast<const uint4*>(gp)[(nb * 32 + lane) * 2 + 1];
                    const uint32_t bw[8] = {f01.x, f01.y, f01.z, f01.w, f23.x, f23.y, f23.z, f23.w};
                    // K steps 0, 1 and 2, 3 as two independent accumulation chains
                    int dk[2][4];
#pragma unroll
                    for (int st = 0; st < 4; ++st) {
                        if (st < 2)
#pragma unroll
                            for (int i = 0; i < 4; ++i) dk[st][i] = 0;
                        const uint32_t a0 = (swA >> st) & 0x01010101u, a2 = (swA >> (st + 4)) & 0x01010101u;
                        const uint32_t a1 = (swB >> st) & 0x01010101u, a3 = (swB >> (st + 4)) & 0x01010101u;
                        mma_s8(dk[st & 1], a0, a1, a2, a3, bw[2 * st], bw[2 * st + 1]);
                    }
#pragma unroll
                    for (int i = 0; i < 4; ++i) dacc[nb][i] = dk[0][i] + dk[1][i];
                }
                const float4* ft = reinterpret_cast<const float4*>(gp + NB * 4 * 256);
#pragma unroll
                for (int nb = 0; nb < NB; ++nb) {
                    const float4 f = ft[nb * 4 + q];                 // factor pair, term pair
                    acc[nb][0] = fmaf(scA, fmaf(f.x, i2f_small(dacc[nb][0]), -f.z), acc[nb][0]);
                    acc[nb][1] = fmaf(scA, fmaf(f.y, i2f_small(dacc[nb][1]), -f.w), acc[nb][1]);
                    acc[nb][2] = fmaf(scB, fmaf(f.x, i2f_small(dacc[nb][2]), -f.z), acc[nb][2]);
                    acc[nb][3] = fmaf(scB, fmaf(f.y, i2f_small(dacc[nb][3]), -f.w), acc[nb][3]);
                }
            }
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(&empty[s]);
            if (k % nu == nu - 1) flush(k, k / nu);
        }
    }
    // Rank 0 leaves after the other ranks' last stores and arrivals reached it;
    // the other ranks' shared memory is not accessed after their last block.
}

// ---------------------------------------------------------------------------
// host
// ---------------------------------------------------------------------------
// tensor maps of recently used weight matrices: (base, rows, row bytes) -> map
struct Q1MapCache {
    struct Entry {
        const void* base = nullptr;
        int rows = 0, rowbytes = 0;
        CUtensorMap map;
    };
    Entry e[32];
    int next = 0;
};

void free_q1_maps(dz_ctx* ctx) {
    delete static_cast<Q1MapCache*>(ctx->q1_maps);
    ctx->q1_maps = nullptr;
}

static bool q1_map(dz_ctx* ctx, const uint8_t* base, int rows, int rowbytes, CUtensorMap* out) {
    if (!ctx->q1_maps) ctx->q1_maps = new Q1MapCache();
    Q1MapCache* cache = static_cast<Q1MapCache*>(ctx->q1_maps);
    for (auto& en : cache->e)
        if (en.base == base && en.rows == rows && en.rowbytes == rowbytes) {
            *out = en.map;
            return true;
        }
    EncodeTiledFn fn = tensor_map_encoder();
    if (!fn) return false;
    cuuint64_t dims[2] = {(cuuint64_t)rowbytes, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)rowbytes};
    cuuint32_t box[2] = {(cuuint32_t)q1::UNIT_BYTES, (cuuint32_t)q1::ROWS};
    cuuint32_t estr[2] = {1, 1};
    Q1MapCache::Entry& en = cache->e[cache->next];
    if (fn(&en.map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(base), dims, strides, box, estr,
           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS) {
        en.base = nullptr;
        return false;
    }
    en.base = base;
    en.rows = rows;
    en.rowbytes = rowbytes;
    cache->next = (cache->next + 1) % 32;
    *out = en.map;
    return true;
}

template <int NB>
static cudaError_t launch_gemv(const Q1Desc& d, int G, size_t smem, const unsigned char* prep, int* err,
                               cudaStream_t st) {
    auto kern = q1_gemv_kernel<NB>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    cudaLaunchAttribute at[2];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    at[1].id = cudaLaunchAttributeClusterDimension;
    at[1].val.clusterDim.x = (unsigned)d.ks;
    at[1].val.clusterDim.y = 1;
    at[1].val.clusterDim.z = 1;
    cudaLaunchConfig_t lc{};
    lc.gridDim = dim3(G);
    lc.blockDim = dim3(q1::THREADS);
    lc.dynamicSmemBytes = smem;
    lc.stream = st;
    lc.attrs = at;
    lc.numAttrs = 2;
    return cudaLaunchKernelEx(&lc, kern, d, prep, err);
}

// CTAs per cluster for nblk row blocks of U units on `slots` resident CTAs: the
// fewest items per CTA, ceil(nblk / clusters) * ceil(U / ks), smallest ks on ties
static int q1_pick_ks(int nblk, int U, int slots) {
    int best = 1;
    long best_items = -1;
    for (int ks = 1; ks <= std::min(Q1_MAX_KS, U); ks *= 2) {
        const int nclus = std::max(1, std::min(nblk, slots / ks));
        // + one item's time for the cross-CTA reduction of a cluster
        const long items = (long)((nblk + nclus - 1) / nclus) * ((U + ks - 1) / ks) + (ks > 1 ? 1 : 0);
        if (best_items < 0 || items < best_items) {
            best_items = items;
            best = ks;
        }
    }
    return best;
}

cudaError_t launch_q1_gemv(dz_ctx* ctx, int n_mats, const uint8_t* const* w, const int32_t* rows, int cols, int T,
                           const float* x, float* const* y, bool accumulate, cudaStream_t st, int* n_launch) {
    const int groups = cols / 128;
    const size_t need = (size_t)groups * q1_group_bytes(T);
    cudaError_t e = ensure_q1_scratch(ctx, need);
    if (e != cudaSuccess) return e;
    unsigned char* prep = static_cast<unsigned char*>(ctx->q1);
    Q1Desc d{};
    d.n_mats = n_mats;
    d.cols = cols;
    d.T = T;
    d.accumulate = accumulate ? 1 : 0;
    d.units = groups / q1::UNIT;
    d.blk0[0] = 0;
    for (int m = 0; m < n_mats; ++m) {
        if (!q1_map(ctx, w[m], rows[m], groups * 18, &d.map[m])) return cudaErrorInvalidValue;
        d.y[m] = y[m];
        d.rows[m] = rows[m];
        d.blk0[m + 1] = d.blk0[m] + (rows[m] + q1::ROWS - 1) / q1::ROWS;
    }
    for (int m = n_mats; m < Q1_MAX_MATS; ++m) d.blk0[m + 1] = d.blk0[n_mats];
    const int nblk = d.blk0[n_mats];
    const int slots = q1::CTAS_PER_SM * ctx->n_sm;
    d.ks = q1_pick_ks(nblk, d.units, slots);
    const int nclus = std::max(1, std::min(nblk, slots / d.ks));
    const int G = nclus * d.ks;
    const size_t smem = q1_smem_bytes(cols, T) - (size_t)(Q1_MAX_KS - d.ks) * q1::ROWS * T * 4;
    {
        // a programmatic dependent of whatever precedes it on the stream (it waits for
        // that grid inside), so the GEMV's weight loads can start while it finishes
        cudaLaunchAttribute at[1];
        at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        at[0].val.programmaticStreamSerializationAllowed = 1;
        cudaLaunchConfig_t lc{};
        lc.gridDim = dim3((groups + q1::PREP_WARPS - 1) / q1::PREP_WARPS, T);
        lc.blockDim = dim3(32 * q1::PREP_WARPS);
        lc.stream = st;
        lc.attrs = at;
        lc.numAttrs = 1;
        if ((e = cudaLaunchKernelEx(&lc, q1_prep_kernel, x, cols, T, prep)) != cudaSuccess) return e;
    }
    const int NB = q1_nb(T);
    if (NB == 1) e = launch_gemv<1>(d, G, smem, prep, ctx->d_err, st);
    else if (NB == 2) e = launch_gemv<2>(d, G, smem, prep, ctx->d_err, st);
    else e = launch_gemv<3>(d, G, smem, prep, ctx->d_err, st);
    if (e != cudaSuccess) return e;
    *n_launch += 2;
    return cudaGetLastError();
}

}  // namespace dz
