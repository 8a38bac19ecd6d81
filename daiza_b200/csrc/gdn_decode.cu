// gdn_decode.cu -- Gated DeltaNet decode step.
//
// Reference: Daiza-engine/src/model/ssm.rs:466-611 (ssm_forward_into after the
// projection GEMV).  Two launch shapes, chosen by how many (sequence, v head)
// tiles the batch has:
//
// Throughput path (many tiles, e.g. 64 sequences x 48 heads), two kernels:
//   1. gdn_dec_prep  (CTA per sequence x 8 channel groups): ring conv1d + SiLU,
//      L2 norms, q scale -> normalised q/k per k head and v per v head; silu(z)
//      and gates; the ring slot `head` receives the raw input row.
//   2. gdn_dec_state (persistent, 3 CTAs per SM, launched as a programmatic
//      dependent of 1): brings each head's 64 KB [128 v][128 k] state tile and
//      its q/k/record rows in with bulk async copies, runs the reference's fused
//      row pass out of shared memory (decay, kv = S k, delta, rank-1 update,
//      y = S q), writes the rows back from registers, then the gated RMSNorm
//      output; the next tile streams in under the epilogue.
//
// Latency path (few tiles, e.g. one sequence), one kernel, gdn_dec_kernel:
//   RS CTAs (a thread-block cluster) share a v head, each owning ROWS = 128/RS
//   rows of the state tile.  Thread 0 starts the bulk copy of the CTA's slice
//   first; meanwhile the warps run the same prologue as gdn_dec_prep for the
//   head's q/k channels and the slice's v channels; then the row pass, and the
//   gated RMSNorm with the RS partial sums of y^2 exchanged through
//   distributed shared memory.  A single sequence spreads over 192 CTAs
//   instead of 48, and there is no second launch.
//
// Either way, state traffic is exactly one read and one write of each tile.
#include <cstddef>

#include "dz_internal.h"

namespace dz {
// gdn_dec_prep writes, per sequence b:
//   qk  [b][32][128]  normalised q (rows 0..15, * 1/sqrt(128)) and k (rows 16..31) of every k head
//   rec [b*vc + vl][264] = v (conv + SiLU) | silu(z) | decay, beta (+6 pad)
constexpr int REC_F = 2 * SSM_D + 8;   // 264 floats (1056 B, 16-byte multiple)
constexpr int PREP_GROUPS = 8;         // 128-channel groups per prep CTA (one per warp)

// ---------------------------------------------------------------------------
// 1. prep: grid (B, chunks of 8 channel groups + 1).  Groups 0..15 are the q
//    channels of k head g, 16..31 the k channels, 32.. the v channels of the
//    local v heads: ring conv1d + SiLU (the reference's tap and FMA order,
//    ssm.rs:492-513), L2 norms (eps on the sum), q scale; the ring slot `head`
//    (the oldest, read by nobody this step) receives the raw row.  The last
//    chunk computes silu(z) and the gates decay = exp(ssm_a * softplus(alpha +
//    dt_bias)), beta = sigmoid(b).
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) gdn_dec_prep_kernel(GdnDecodeDesc d, int vh0, int vc,
                                                           const SsmSlot* __restrict__ ssm,
                                                           const float* __restrict__ conv_w,
                                                           const float* __restrict__ ssm_a,
                                                           const float* __restrict__ dt_bias,
                                                           const float* __restrict__ qkv,
                                                           const float* __restrict__ alpha_in,
                                                           const float* __restrict__ beta_in,
                                                           const float* __restrict__ z_in, float* __restrict__ qk,
                                                           float* __restrict__ rec) {
    // a programmatic dependent of whatever precedes it: wait for that grid (the
    // states and rings may still be in use by it), then let the state kernel start
    // its tile copies; it waits for this grid's writes before reading q/k/records
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;");
    const int b = blockIdx.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n_groups = 2 * SSM_HK + vc;
    const int n_chunks = (n_groups + PREP_GROUPS - 1) / PREP_GROUPS;
    if ((int)blockIdx.y == n_chunks) {
        // silu(z) and gates for every local v head
        for (int vl = warp; vl < vc; vl += 8) {
            const int vh = vh0 + vl;
            float* r = rec + ((size_t)b * vc + vl) * REC_F;
            const float4 zz = *reinterpret_cast<const float4*>(z_in + (size_t)b * INNER + (size_t)vh * SSM_D + 4 * lane);
            *reinterpret_cast<float4*>(r + SSM_D + 4 * lane) =
                make_float4(siluf_acc(zz.x), siluf_acc(zz.y), siluf_acc(zz.z), siluf_acc(zz.w));
            if (lane == 0) {
                const float g = ssm_a[vh] * softplus_ref(alpha_in[(size_t)b * SSM_HV + vh] + dt_bias[vh]);
                r[2 * SSM_D] = expf(g);
                r[2 * SSM_D + 1] = sigmoidf_acc(beta_in[(size_t)b * SSM_HV + vh]);
            }
        }
        return;
    }
    const int gi = blockIdx.y * PREP_GROUPS + warp;
    if (gi >= n_groups) return;
    const SsmSlot slot = ssm[d.sid[b]];
    float* hist = slot.hist;
    const int head = d.head[b];
    const int r0 = (head + 1) & 3, r1 = (head + 2) & 3, r2 = (head + 3) & 3;
    const float* row_in = qkv + (size_t)b * QKV_LEN;
    int cb;
    if (gi < SSM_HK) cb = gi * SSM_D;
    else if (gi < 2 * SSM_HK) cb = QKD + (gi - SSM_HK) * SSM_D;
    else cb = 2 * QKD + (vh0 + gi - 2 * SSM_HK) * SSM_D;
    const int ch = cb + 4 * lane;
    const float4 h0 = *reinterpret_cast<const float4*>(hist + (size_t)r0 * QKV_LEN + ch);
    const float4 h1 = *reinterpret_cast<const float4*>(hist + (size_t)r1 * QKV_LEN + ch);
    const float4 h2 = *reinterpret_cast<const float4*>(hist + (size_t)r2 * QKV_LEN + ch);
    const float4 cur = *reinterpret_cast<const float4*>(row_in + ch);
    const float4 w0 = *reinterpret_cast<const float4*>(conv_w + 0 * QKV_LEN + ch);
    const float4 w1 = *reinterpret_cast<const float4*>(conv_w + 1 * QKV_LEN + ch);
    const float4 w2 = *reinterpret_cast<const float4*>(conv_w + 2 * QKV_LEN + ch);
    const float4 w3 = *reinterpret_cast<const float4*>(conv_w + 3 * QKV_LEN + ch);
    float4 a;
    a.x = fmaf(cur.x, w3.x, fmaf(h2.x, w2.x, fmaf(h1.x, w1.x, fmaf(h0.x, w0.x, 0.0f))));
    a.y = fmaf(cur.y, w3.y, fmaf(h2.y, w2.y, fmaf(h1.y, w1.y, fmaf(h0.y, w0.y, 0.0f))));
    a.z = fmaf(cur.z, w3.z, fmaf(h2.z, w2.z, fmaf(h1.z, w1.z, fmaf(h0.z, w0.z, 0.0f))));
    a.w = fmaf(cur.w, w3.w, fmaf(h2.w, w2.w, fmaf(h1.w, w1.w, fmaf(h0.w, w0.w, 0.0f))));
    a = make_float4(siluf_acc(a.x), siluf_acc(a.y), siluf_acc(a.z), siluf_acc(a.w));
    bool write_ring;
    if (gi < 2 * SSM_HK) {
        const float ss = warp_sum(a.x * a.x + a.y * a.y + a.z * a.z + a.w * a.w);
        const float inv = 1.0f / sqrtf(ss + 1e-6f);
        a = make_float4(a.x * inv, a.y * inv, a.z * inv, a.w * inv);
        if (gi < SSM_HK) {
            const float qs = 1.0f / sqrtf((float)SSM_D);
            a = make_float4(a.x * qs, a.y * qs, a.z * qs, a.w * qs);
        }
        *reinterpret_cast<float4*>(qk + ((size_t)b * 2 * SSM_HK + gi) * SSM_D + 4 * lane) = a;
        const int kh = gi % SSM_HK;
        // the ring keeps q/k channels of k heads some local v head uses
        const int first = vh0 + (((kh - vh0) % SSM_HK) + SSM_HK) % SSM_HK;
        write_ring = first < vh0 + vc;
    } else {
        const int vl = gi - 2 * SSM_HK;
        *reinterpret_cast<float4*>(rec + ((size_t)b * vc + vl) * REC_F + 4 * lane) = a;
        write_ring = true;
    }
    if (write_ring) *reinterpret_cast<float4*>(hist + (size_t)head * QKV_LEN + ch) = cur;
}

// ---------------------------------------------------------------------------
// 2. state pass: persistent CTAs (STATE_CPS per SM, 8 warps each) walk their
//    items (sequence, v head); per item one bulk copy brings the 64 KB
//    [128 v][128 k] tile and the q/k/record rows into shared memory.  The row
//    pass follows the reference's fused update (ssm.rs:390-417): S *= decay,
//    kv = S k, delta = (v - kv) beta, S += k delta^T, y = S q.  A warp takes 4
//    rows at a time, 8 lanes per row (16 columns each, three shuffle levels per
//    dot product), and stores the updated rows straight from registers.  The
//    next item's copy is issued as soon as the tile is consumed, under the
//    gated RMSNorm output (ssm.rs:576-611).  The first tile is requested before
//    the programmatic-dependency wait, so it streams in while gdn_dec_prep is
//    still finishing.
// ---------------------------------------------------------------------------
constexpr int STATE_CPS = 3;   // resident CTAs per SM (3 x 67 KB shared memory)
struct alignas(128) RecBuf {
    float q[SSM_D], k[SSM_D];
    float r[REC_F];            // v | silu(z) | decay, beta
};
struct GdnSmem {
    float S[SSM_D][SSM_D];     // 64 KB
    RecBuf rec[2];
    float y[SSM_D];
    float red[8];
    uint64_t full;
};
static_assert(offsetof(GdnSmem, rec) % 16 == 0 && sizeof(RecBuf) % 16 == 0 && offsetof(RecBuf, k) % 16 == 0 &&
                  offsetof(RecBuf, r) % 16 == 0,
              "bulk-copy alignment");

__global__ void __launch_bounds__(256, STATE_CPS) gdn_dec_state_kernel(GdnDecodeDesc d, int vh0, int vc,
                                                                      const SsmSlot* __restrict__ ssm,
                                                                      const float* __restrict__ norm_w,
                                                                      const float* __restrict__ qk,
                                                                      const float* __restrict__ rec,
                                                                      float* __restrict__ y_out, int n_items,
                                                                      int* err) {
    extern __shared__ __align__(128) unsigned char smem_raw[];
    GdnSmem& sm = *reinterpret_cast<GdnSmem*>(smem_raw);
    asm volatile("griddepcontrol.launch_dependents;");
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 3, c = lane & 7;   // row within a 4-row group, column lane
    auto state_ptr = [&](int item) {
        const int b = item / vc, vl = item - b * vc;
        return ssm[d.sid[b]].state + (size_t)vl * SSM_D * SSM_D;
    };
    constexpr uint32_t TILE_BYTES = SSM_D * SSM_D * 4;
    constexpr uint32_t REC_BYTES = 2 * SSM_D * 4 + REC_F * 4;
    auto issue_records = [&](int item, int slot) {
        const int b = item / vc, kh = (vh0 + item - b * vc) % SSM_HK;
        RecBuf& R = sm.rec[slot];
        bulk_g2s(&R.q[0], qk + ((size_t)b * 2 * SSM_HK + kh) * SSM_D, SSM_D * 4, &sm.full);
        bulk_g2s(&R.k[0], qk + ((size_t)b * 2 * SSM_HK + SSM_HK + kh) * SSM_D, SSM_D * 4, &sm.full);
        bulk_g2s(&R.r[0], rec + (size_t)item * REC_F, REC_F * 4, &sm.full);
    };
    if (tid == 0) {
        mbar_init(&sm.full, 1);
        fence_mbar_init();
        if ((int)blockIdx.x < n_items) {
            mbar_arrive_expect_tx(&sm.full, TILE_BYTES + REC_BYTES);
            bulk_g2s(&sm.S[0][0], state_ptr(blockIdx.x), TILE_BYTES, &sm.full);
        }
    }
    // q/k/records come from gdn_dec_prep
    asm volatile("griddepcontrol.wait;" ::: "memory");
    if (tid == 0 && (int)blockIdx.x < n_items) issue_records(blockIdx.x, 0);
    __syncthreads();
    const float nw = norm_w[tid & (SSM_D - 1)];
    int k = 0;
    for (int item = blockIdx.x; item < n_items; item += gridDim.x, ++k) {
        if (!mbar_wait(&sm.full, (uint32_t)(k & 1), err)) return;
        const RecBuf& R = sm.rec[k & 1];
        float* gS = state_ptr(item);
        const float decay = R.r[2 * SSM_D], beta = R.r[2 * SSM_D + 1];
        float4 kq[4], qq[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            kq[j] = *reinterpret_cast<const float4*>(&R.k[32 * j + 4 * c]);
            qq[j] = *reinterpret_cast<const float4*>(&R.q[32 * j + 4 * c]);
        }
#pragma unroll 2
        for (int it = 0; it < 4; ++it) {
            const int i = 16 * warp + 4 * it + g;
            float4 sv[4];
            float kv = 0.0f;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                sv[j] = *reinterpret_cast<const float4*>(&sm.S[i][32 * j + 4 * c]);
                sv[j].x *= decay; sv[j].y *= decay; sv[j].z *= decay; sv[j].w *= decay;
                kv = fmaf(sv[j].x, kq[j].x, kv);
                kv = fmaf(sv[j].y, kq[j].y, kv);
                kv = fmaf(sv[j].z, kq[j].z, kv);
                kv = fmaf(sv[j].w, kq[j].w, kv);
            }
            kv += __shfl_xor_sync(0xffffffffu, kv, 1);
            kv += __shfl_xor_sync(0xffffffffu, kv, 2);
            kv += __shfl_xor_sync(0xffffffffu, kv, 4);
            const float di = (R.r[i] - kv) * beta;
            float yy = 0.0f;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                sv[j].x = fmaf(di, kq[j].x, sv[j].x);
                sv[j].y = fmaf(di, kq[j].y, sv[j].y);
                sv[j].z = fmaf(di, kq[j].z, sv[j].z);
                sv[j].w = fmaf(di, kq[j].w, sv[j].w);
                yy = fmaf(sv[j].x, qq[j].x, yy);
                yy = fmaf(sv[j].y, qq[j].y, yy);
                yy = fmaf(sv[j].z, qq[j].z, yy);
                yy = fmaf(sv[j].w, qq[j].w, yy);
                // the next read of this state is a whole layer stack away: streaming store
                __stcs(reinterpret_cast<float4*>(gS + (size_t)i * SSM_D + 32 * j + 4 * c), sv[j]);
            }
            yy += __shfl_xor_sync(0xffffffffu, yy, 1);
            yy += __shfl_xor_sync(0xffffffffu, yy, 2);
            yy += __shfl_xor_sync(0xffffffffu, yy, 4);
            if (c == 0) sm.y[i] = yy;
        }
        __syncthreads();   // tile consumed, y complete
        const int nxt = item + gridDim.x;
        if (tid == 0 && nxt < n_items) {
            mbar_arrive_expect_tx(&sm.full, TILE_BYTES + REC_BYTES);
            bulk_g2s(&sm.S[0][0], state_ptr(nxt), TILE_BYTES, &sm.full);
            issue_records(nxt, (k + 1) & 1);
        }
        // gated RMSNorm: threads 0..127 own one element of y
        float yv = 0.0f;
        if (tid < SSM_D) yv = sm.y[tid];
        float ss = warp_sum(yv * yv);
        if (lane == 0) sm.red[warp] = ss;
        __syncthreads();
        if (tid < SSM_D) {
            ss = sm.red[0] + sm.red[1] + sm.red[2] + sm.red[3];
            const float inv = 1.0f / sqrtf(ss * (1.0f / (float)SSM_D) + 1e-6f);
            y_out[(size_t)item * SSM_D + tid] = ((yv * inv) * nw) * R.r[SSM_D + tid];
        }
        __syncthreads();   // y, red and this record slot are reused two items on
    }
}


// ---------------------------------------------------------------------------
// latency path: one fused kernel per (sequence, v head, row slice)
// ---------------------------------------------------------------------------

template <int RS>
struct GdnDecSmem {
    static constexpr int ROWS = SSM_D / RS;
    float S[ROWS][SSM_D];      // state rows [r0, r0 + ROWS)
    float q[SSM_D], k[SSM_D];  // normalised q (scaled) and k of the head's k head
    float v[ROWS];             // conv + SiLU v channels of the slice
    float zs[ROWS];            // silu(z) of the slice
    float y[ROWS];
    float gate[2];             // decay, beta
    float ss_part;             // this CTA's sum of y^2 (read by the cluster)
    float inv_rms;
    uint64_t full;
};

__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// load a float from the shared memory of CTA `rank` of this cluster
__device__ __forceinline__ float ld_cluster_f32(const float* p, uint32_t rank) {
    uint32_t remote;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(smem_u32(p)), "r"(rank));
    float v;
    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(remote) : "memory");
    return v;
}

// conv1d over the ring (the reference's tap order, ssm.rs:492-513) + SiLU
__device__ __forceinline__ float conv_silu(float h0, float h1, float h2, float cur, float w0, float w1, float w2,
                                           float w3) {
    return siluf_acc(fmaf(cur, w3, fmaf(h2, w2, fmaf(h1, w1, fmaf(h0, w0, 0.0f)))));
}

template <int RS>
__global__ void __launch_bounds__(32 * (SSM_D / RS / 8)) gdn_dec_kernel(
    GdnDecodeDesc d, int vh0, int vc, const SsmSlot* __restrict__ ssm, const float* __restrict__ conv_w,
    const float* __restrict__ ssm_a, const float* __restrict__ dt_bias, const float* __restrict__ norm_w,
    const float* __restrict__ qkv, const float* __restrict__ alpha_in, const float* __restrict__ beta_in,
    const float* __restrict__ z_in, float* __restrict__ y_out, int* err) {
    using Smem = GdnDecSmem<RS>;
    constexpr int ROWS = Smem::ROWS;
    extern __shared__ __align__(128) unsigned char smem_raw[];
    Smem& sm = *reinterpret_cast<Smem*>(smem_raw);
    // launched as a programmatic dependent of whatever precedes it: wait for that
    // grid (the state may still be in use by it) before anything else; then a
    // programmatic successor (the next projection) may start streaming its weights
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;");
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int item = blockIdx.x / RS;                 // b * vc + vl
    const int rank = (int)cluster_rank();             // == blockIdx.x % RS
    const int b = item / vc, vl = item - b * vc, vh = vh0 + vl, kh = vh % SSM_HK;   // ssm.rs:558-561
    const int r0 = rank * ROWS;
    const SsmSlot slot = ssm[d.sid[b]];
    float* gS = slot.state + ((size_t)vl * SSM_D + r0) * SSM_D;

    if (tid == 0) {
        mbar_init(&sm.full, 1);
        fence_mbar_init();
        mbar_arrive_expect_tx(&sm.full, ROWS * SSM_D * 4);
        bulk_g2s(&sm.S[0][0], gS, ROWS * SSM_D * 4, &sm.full);
    }

    // ---- prologue (ssm.rs:466-540)
    float* hist = slot.hist;
    const int head = d.head[b];
    const float* h0p = hist + (size_t)((head + 1) & 3) * QKV_LEN;   // oldest of the three kept rows
    const float* h1p = hist + (size_t)((head + 2) & 3) * QKV_LEN;
    const float* h2p = hist + (size_t)((head + 3) & 3) * QKV_LEN;
    float* hw = hist + (size_t)head * QKV_LEN;                       // slot receiving the current row
    const float* row_in = qkv + (size_t)b * QKV_LEN;
    if (warp < 2) {
        // warp 0: q channels of k head kh, warp 1: its k channels; lane owns 4 channels
        const int ch = (warp == 0 ? 0 : QKD) + kh * SSM_D + 4 * lane;
        const float4 a0 = *reinterpret_cast<const float4*>(h0p + ch);
        const float4 a1 = *reinterpret_cast<const float4*>(h1p + ch);
        const float4 a2 = *reinterpret_cast<const float4*>(h2p + ch);
        const float4 cur = *reinterpret_cast<const float4*>(row_in + ch);
        const float4 w0 = *reinterpret_cast<const float4*>(conv_w + 0 * QKV_LEN + ch);
        const float4 w1 = *reinterpret_cast<const float4*>(conv_w + 1 * QKV_LEN + ch);
        const float4 w2 = *reinterpret_cast<const float4*>(conv_w + 2 * QKV_LEN + ch);
        const float4 w3 = *reinterpret_cast<const float4*>(conv_w + 3 * QKV_LEN + ch);
        float4 a;
        a.x = conv_silu(a0.x, a1.x, a2.x, cur.x, w0.x, w1.x, w2.x, w3.x);
        a.y = conv_silu(a0.y, a1.y, a2.y, cur.y, w0.y, w1.y, w2.y, w3.y);
        a.z = conv_silu(a0.z, a1.z, a2.z, cur.z, w0.z, w1.z, w2.z, w3.z);
        a.w = conv_silu(a0.w, a1.w, a2.w, cur.w, w0.w, w1.w, w2.w, w3.w);
        const float ss = warp_sum(a.x * a.x + a.y * a.y + a.z * a.z + a.w * a.w);
        const float inv = 1.0f / sqrtf(ss + 1e-6f);                    // l2norm_inplace, ssm.rs:76-135
        a = make_float4(a.x * inv, a.y * inv, a.z * inv, a.w * inv);
        if (warp == 0) {
            const float qs = 1.0f / sqrtf((float)SSM_D);                 // ssm.rs:531-533
            a = make_float4(a.x * qs, a.y * qs, a.z * qs, a.w * qs);
            *reinterpret_cast<float4*>(&sm.q[4 * lane]) = a;
        } else {
            *reinterpret_cast<float4*>(&sm.k[4 * lane]) = a;
        }
        // one writer per q/k ring channel: the first local v head of this k head, slice 0
        const int first = vh0 + (((kh - vh0) % SSM_HK) + SSM_HK) % SSM_HK;
        if (vh == first && rank == 0) *reinterpret_cast<float4*>(hw + ch) = cur;
    } else if (warp == 2) {
        // v channels of the slice
        for (int r = lane; r < ROWS; r += 32) {
            const int ch = 2 * QKD + vh * SSM_D + r0 + r;
            const float cur = row_in[ch];
            sm.v[r] = conv_silu(h0p[ch], h1p[ch], h2p[ch], cur, conv_w[ch], conv_w[QKV_LEN + ch],
                                conv_w[2 * QKV_LEN + ch], conv_w[3 * QKV_LEN + ch]);
            hw[ch] = cur;
        }
    } else if (warp == 3) {
        for (int r = lane; r < ROWS; r += 32) sm.zs[r] = siluf_acc(z_in[(size_t)b * INNER + (size_t)vh * SSM_D + r0 + r]);
        if (lane == 0) {
            const float g = ssm_a[vh] * softplus_ref(alpha_in[(size_t)b * SSM_HV + vh] + dt_bias[vh]);   // ssm.rs:535-540
            sm.gate[0] = expf(g);
            sm.gate[1] = sigmoidf_acc(beta_in[(size_t)b * SSM_HV + vh]);
        }
    }
    __syncthreads();

    // ---- row pass (ssm.rs:390-417): warp w owns rows [8w, 8w+8), 4 at a time
    const bool ok = mbar_wait(&sm.full, 0, err);
    if (ok) {
        const int g = lane >> 3, c = lane & 7;
        const float decay = sm.gate[0], beta = sm.gate[1];
        float4 kq[4], qq[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            kq[j] = *reinterpret_cast<const float4*>(&sm.k[32 * j + 4 * c]);
            qq[j] = *reinterpret_cast<const float4*>(&sm.q[32 * j + 4 * c]);
        }
#pragma unroll
        for (int it = 0; it < 2; ++it) {
            const int i = 8 * warp + 4 * it + g;
            float4 sv[4];
            float kv = 0.0f;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                sv[j] = *reinterpret_cast<const float4*>(&sm.S[i][32 * j + 4 * c]);
                sv[j].x *= decay; sv[j].y *= decay; sv[j].z *= decay; sv[j].w *= decay;
                kv = fmaf(sv[j].x, kq[j].x, kv);
                kv = fmaf(sv[j].y, kq[j].y, kv);
                kv = fmaf(sv[j].z, kq[j].z, kv);
                kv = fmaf(sv[j].w, kq[j].w, kv);
            }
            kv += __shfl_xor_sync(0xffffffffu, kv, 1);
            kv += __shfl_xor_sync(0xffffffffu, kv, 2);
            kv += __shfl_xor_sync(0xffffffffu, kv, 4);
            const float di = (sm.v[i] - kv) * beta;
            float yy = 0.0f;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                sv[j].x = fmaf(di, kq[j].x, sv[j].x);
                sv[j].y = fmaf(di, kq[j].y, sv[j].y);
                sv[j].z = fmaf(di, kq[j].z, sv[j].z);
                sv[j].w = fmaf(di, kq[j].w, sv[j].w);
                yy = fmaf(sv[j].x, qq[j].x, yy);
                yy = fmaf(sv[j].y, qq[j].y, yy);
                yy = fmaf(sv[j].z, qq[j].z, yy);
                yy = fmaf(sv[j].w, qq[j].w, yy);
                // the next read of this state is a whole layer stack away: streaming store
                __stcs(reinterpret_cast<float4*>(gS + (size_t)i * SSM_D + 32 * j + 4 * c), sv[j]);
            }
            yy += __shfl_xor_sync(0xffffffffu, yy, 1);
            yy += __shfl_xor_sync(0xffffffffu, yy, 2);
            yy += __shfl_xor_sync(0xffffffffu, yy, 4);
            if (c == 0) sm.y[i] = yy;
        }
    }
    __syncthreads();
    if (warp == 0) {
        float s = 0.0f;
        for (int r = lane; r < ROWS; r += 32) s += sm.y[r] * sm.y[r];
        s = warp_sum(s);
        if (lane == 0) sm.ss_part = s;
    }
    // ---- gated RMSNorm across the cluster.  Every CTA passes both cluster
    // barriers, also after a failed wait, so no CTA of the cluster is left behind.
    cluster_sync_all();
    if (tid == 0) {
        float ss = 0.0f;
#pragma unroll
        for (int r = 0; r < RS; ++r) ss += ld_cluster_f32(&sm.ss_part, (uint32_t)r);
        sm.inv_rms = 1.0f / sqrtf(ss * (1.0f / (float)SSM_D) + 1e-6f);
    }
    cluster_sync_all();   // partials read before any CTA of the cluster exits; inv_rms visible
    if (ok && tid < ROWS)
        y_out[(size_t)item * SSM_D + r0 + tid] = ((sm.y[tid] * sm.inv_rms) * norm_w[r0 + tid]) * sm.zs[tid];
}

static cudaError_t launch_two_pass(dz_ctx* ctx, int layer, const GdnDecodeDesc& d, const float* qkv,
                                  const float* alpha, const float* beta, const float* z, float* y,
                                  cudaStream_t st, int* n_launch) {
    const LayerState& L = ctx->layers[layer];
    const int vc = ctx->cfg.v_head_count, vh0 = ctx->cfg.v_head_begin;
    const int items = d.B * vc;
    const size_t qk_floats = (size_t)d.B * 2 * SSM_HK * SSM_D;
    cudaError_t e = ensure_decode_records(ctx, (qk_floats + (size_t)items * REC_F) * sizeof(float));
    if (e != cudaSuccess) return e;
    float* qk = ctx->gdn_rec;
    float* rec = qk + qk_floats;
    const int n_chunks = (2 * SSM_HK + vc + PREP_GROUPS - 1) / PREP_GROUPS;
    {
        cudaLaunchAttribute ap[1];
        ap[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        ap[0].val.programmaticStreamSerializationAllowed = 1;
        cudaLaunchConfig_t lp{};
        lp.gridDim = dim3(d.B, n_chunks + 1);
        lp.blockDim = dim3(256);
        lp.stream = st;
        lp.attrs = ap;
        lp.numAttrs = 1;
        e = cudaLaunchKernelEx(&lp, gdn_dec_prep_kernel, d, vh0, vc, (const SsmSlot*)L.d_ssm, (const float*)L.conv_w,
                               (const float*)L.ssm_a, (const float*)L.dt_bias, qkv, alpha, beta, z, qk, rec);
        if (e != cudaSuccess) return e;
    }
    e = cudaFuncSetAttribute(gdn_dec_state_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(GdnSmem));
    if (e != cudaSuccess) return e;
    // programmatic dependent launch: the state kernel's CTAs start their first
    // tile copy while the prep grid drains
    cudaLaunchConfig_t lc{};
    lc.gridDim = dim3(items < ctx->n_sm * STATE_CPS ? items : ctx->n_sm * STATE_CPS);
    lc.blockDim = dim3(256);
    lc.dynamicSmemBytes = sizeof(GdnSmem);
    lc.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    lc.attrs = at;
    lc.numAttrs = 1;
    e = cudaLaunchKernelEx(&lc, gdn_dec_state_kernel, d, vh0, vc, (const SsmSlot*)L.d_ssm, (const float*)L.norm_w,
                           (const float*)qk, (const float*)rec, y, items, ctx->d_err);
    *n_launch += 2;
    return e != cudaSuccess ? e : cudaGetLastError();
}


template <int RS>
static cudaError_t launch_rs(dz_ctx* ctx, const LayerState& L, const GdnDecodeDesc& d, int vh0, int vc,
                             const float* qkv, const float* alpha, const float* beta, const float* z, float* y,
                             cudaStream_t st) {
    auto kern = gdn_dec_kernel<RS>;
    const int smem = (int)sizeof(GdnDecSmem<RS>);
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t lc{};
    lc.gridDim = dim3(d.B * vc * RS);
    lc.blockDim = dim3(32 * (SSM_D / RS / 8));
    lc.dynamicSmemBytes = smem;
    lc.stream = st;
    cudaLaunchAttribute at[2];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = RS;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[1].val.programmaticStreamSerializationAllowed = 1;
    lc.attrs = at;
    lc.numAttrs = 2;
    return cudaLaunchKernelEx(&lc, kern, d, vh0, vc, (const SsmSlot*)L.d_ssm, (const float*)L.conv_w,
                              (const float*)L.ssm_a, (const float*)L.dt_bias, (const float*)L.norm_w, qkv, alpha,
                              beta, z, y, ctx->d_err);
}

cudaError_t launch_gdn_decode(dz_ctx* ctx, int layer, const GdnDecodeDesc& d, const float* qkv,
                              const float* alpha, const float* beta, const float* z, float* y,
                              cudaStream_t st, int* n_launch) {
    const LayerState& L = ctx->layers[layer];
    const int vc = ctx->cfg.v_head_count, vh0 = ctx->cfg.v_head_begin;
    const int heads = d.B * vc;
    // more tiles than two per SM: the persistent two-kernel path keeps HBM busier
    if (heads > 2 * ctx->n_sm) return launch_two_pass(ctx, layer, d, qkv, alpha, beta, z, y, st, n_launch);
    cudaError_t e = launch_rs<4>(ctx, L, d, vh0, vc, qkv, alpha, beta, z, y, st);
    *n_launch += 1;
    return e != cudaSuccess ? e : cudaGetLastError();
}

}  // namespace dz
