// gdn_decode.cu -- Gated DeltaNet decode step.
//
// Reference: Daiza-engine/src/model/ssm.rs:466-611 (ssm_forward_into after the
// projection GEMV).  Two stream-ordered kernels:
//   1. gdn_dec_prep  (CTA per sequence x 8 channel groups): ring conv1d + SiLU,
//      L2 norms, q scale -> normalised q/k per k head and v per v head; silu(z)
//      and gates; the ring slot `head` receives the raw input row.
//   2. gdn_dec_state (persistent, 3 CTAs per SM, launched as a programmatic
//      dependent of 1): brings each head's 64 KB [128 v][128 k] state tile and
//      its q/k/record rows in with bulk async copies, runs the reference's fused
//      row pass out of shared memory (decay, kv = S k, delta, rank-1 update,
//      y = S q), writes the rows back from registers, then the gated RMSNorm
//      output.
// State traffic is exactly one read and one write of each tile.
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
    // the state kernel may start its tile copies now; it waits for this grid's
    // writes before reading q/k/records
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

cudaError_t launch_gdn_decode(dz_ctx* ctx, int layer, const GdnDecodeDesc& d, const float* qkv,
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
    gdn_dec_prep_kernel<<<dim3(d.B, n_chunks + 1), 256, 0, st>>>(d, vh0, vc, L.d_ssm, L.conv_w, L.ssm_a, L.dt_bias,
                                                                qkv, alpha, beta, z, qk, rec);
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

}  // namespace dz
