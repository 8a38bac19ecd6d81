// gdn_decode.cu -- fused Gated DeltaNet decode step.
//
// Reference: Daiza-engine/src/model/ssm.rs:466-611 (ssm_forward_into after the
// projection GEMV).  One CTA per (sequence, v head), 128 threads:
//   - the head's 64 KB state tile is brought into shared memory by four 16 KB
//     bulk async copies (one mbarrier per 32-row quarter) that overlap with
//   - the ring conv1d (k=4) + SiLU of the q/k channels of k head vh % 16 and
//     the v channels of vh, L2-norm of q and k, q *= 1/sqrt(128), the gates
//     decay = exp(ssm_a * softplus(alpha + dt_bias)) and beta = sigmoid(b);
//   - each warp then runs the reference's fused row pass (ssm.rs:378-418) on
//     its 32 rows straight out of shared memory (decay, kv = S k, delta,
//     rank-1 update, y = S q; warp-shuffle dot products) and writes its rows
//     back with one 16 KB bulk store;
//   - the gated RMSNorm output y * inv_rms * w * silu(z) (ssm.rs:576-611).
// State traffic is exactly one read and one write of each tile.
#include <cstddef>

#include "dz_internal.h"

namespace dz {

struct GdnSmem {
    float S[SSM_D][SSM_D];   // 64 KB state tile
    float q[SSM_D], k[SSM_D], v[SSM_D], y[SSM_D];
    float red[3][4];
    float gate[2];           // decay, beta
    uint64_t bar[4];
};
static_assert(offsetof(GdnSmem, q) % 16 == 0 && offsetof(GdnSmem, k) % 16 == 0, "float4-read fields aligned");

__device__ __forceinline__ float block_sum128(float x, float* red4) {
    x = warp_sum(x);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) red4[warp] = x;
    __syncthreads();
    return red4[0] + red4[1] + red4[2] + red4[3];
}

__global__ void __launch_bounds__(128) gdn_decode_kernel(GdnDecodeDesc d, int vh0, const SsmSlot* __restrict__ ssm,
                                                         const float* __restrict__ conv_w,
                                                         const float* __restrict__ ssm_a,
                                                         const float* __restrict__ dt_bias,
                                                         const float* __restrict__ norm_w,
                                                         const float* __restrict__ qkv,
                                                         const float* __restrict__ alpha_in,
                                                         const float* __restrict__ beta_in,
                                                         const float* __restrict__ z_in, float* __restrict__ y_out,
                                                         int vcount, int* err) {
    extern __shared__ __align__(128) unsigned char smem_raw[];
    GdnSmem& sm = *reinterpret_cast<GdnSmem*>(smem_raw);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int vl = blockIdx.x;                 // local v head
    const int vh = vh0 + vl;                   // global v head
    const int b = blockIdx.y;
    const int kh = vh % SSM_HK;                // tiled k-head map (ssm.rs:558-561)
    const SsmSlot slot = ssm[d.sid[b]];
    float* Sg = slot.state + (size_t)vl * SSM_D * SSM_D;
    float* hist = slot.hist;
    const int head = d.head[b];

    if (tid == 0) {
        for (int i = 0; i < 4; ++i) mbar_init(&sm.bar[i], 1);
        fence_mbar_init();
    }
    __syncthreads();
    if (tid == 0) {
        for (int i = 0; i < 4; ++i) {
            mbar_arrive_expect_tx(&sm.bar[i], 32 * SSM_D * 4);
            bulk_g2s(&sm.S[32 * i][0], Sg + (size_t)32 * i * SSM_D, 32 * SSM_D * 4, &sm.bar[i]);
        }
    }

    // ---- conv1d ring + SiLU (ssm.rs:473-518).  Taps t=0..2 are the ring rows
    // (head+1+t)%4 (oldest first), tap 3 is the current token.
    const float* row_in = qkv + (size_t)b * QKV_LEN;
    const int r0 = (head + 1) & 3, r1 = (head + 2) & 3, r2 = (head + 3) & 3;
    const int chq = kh * SSM_D + tid, chk = QKD + kh * SSM_D + tid, chv = 2 * QKD + vh * SSM_D + tid;
    float cq, ck, cv;
    {
        auto conv = [&](int ch) {
            float acc = 0.0f;
            acc = fmaf(hist[(size_t)r0 * QKV_LEN + ch], conv_w[0 * QKV_LEN + ch], acc);
            acc = fmaf(hist[(size_t)r1 * QKV_LEN + ch], conv_w[1 * QKV_LEN + ch], acc);
            acc = fmaf(hist[(size_t)r2 * QKV_LEN + ch], conv_w[2 * QKV_LEN + ch], acc);
            acc = fmaf(row_in[ch], conv_w[3 * QKV_LEN + ch], acc);
            return siluf_acc(acc);
        };
        cq = conv(chq);
        ck = conv(chk);
        cv = conv(chv);
    }
    // ring write of the current row into slot `head` (the oldest; nobody reads it
    // this step).  q/k channels of kh are written by the first local v head that
    // maps to kh; v channels by their own head.
    if (vh - SSM_HK < vh0) {
        hist[(size_t)head * QKV_LEN + chq] = row_in[chq];
        hist[(size_t)head * QKV_LEN + chk] = row_in[chk];
    }
    hist[(size_t)head * QKV_LEN + chv] = row_in[chv];

    // ---- L2 norm (eps on the sum, ssm.rs:123) and q scale
    const float ssq = block_sum128(cq * cq, sm.red[0]);
    const float ssk = block_sum128(ck * ck, sm.red[1]);
    const float qs = 1.0f / sqrtf((float)SSM_D);
    sm.q[tid] = (cq * (1.0f / sqrtf(ssq + 1e-6f))) * qs;
    sm.k[tid] = ck * (1.0f / sqrtf(ssk + 1e-6f));
    sm.v[tid] = cv;
    if (tid == 0) {
        const float g = ssm_a[vh] * softplus_ref(alpha_in[(size_t)b * SSM_HV + vh] + dt_bias[vh]);
        sm.gate[0] = expf(g);
        sm.gate[1] = sigmoidf_acc(beta_in[(size_t)b * SSM_HV + vh]);
    }
    __syncthreads();

    // ---- fused row pass on this warp's 32 rows (ssm.rs:390-417)
    const float decay = sm.gate[0], beta = sm.gate[1];
    const float4 kq = *reinterpret_cast<const float4*>(&sm.k[4 * lane]);
    const float4 qq = *reinterpret_cast<const float4*>(&sm.q[4 * lane]);
    bool ok = mbar_wait(&sm.bar[warp], 0, err);
    if (ok) {
#pragma unroll 4
        for (int r = 0; r < 32; ++r) {
            const int i = 32 * warp + r;
            float4 s = *reinterpret_cast<const float4*>(&sm.S[i][4 * lane]);
            s.x *= decay; s.y *= decay; s.z *= decay; s.w *= decay;
            float kv = s.x * kq.x;
            kv = fmaf(s.y, kq.y, kv);
            kv = fmaf(s.z, kq.z, kv);
            kv = fmaf(s.w, kq.w, kv);
            kv = warp_sum(kv);
            const float di = (sm.v[i] - kv) * beta;
            s.x = fmaf(di, kq.x, s.x);
            s.y = fmaf(di, kq.y, s.y);
            s.z = fmaf(di, kq.z, s.z);
            s.w = fmaf(di, kq.w, s.w);
            float yy = s.x * qq.x;
            yy = fmaf(s.y, qq.y, yy);
            yy = fmaf(s.z, qq.z, yy);
            yy = fmaf(s.w, qq.w, yy);
            yy = warp_sum(yy);
            *reinterpret_cast<float4*>(&sm.S[i][4 * lane]) = s;
            if (lane == 0) sm.y[i] = yy;
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
            bulk_s2g(Sg + (size_t)32 * warp * SSM_D, &sm.S[32 * warp][0], 32 * SSM_D * 4);
            bulk_commit();
        }
    }
    __syncthreads();

    // ---- gated RMSNorm output (ssm.rs:576-611): y * inv_rms * w * silu(z)
    const float yv = sm.y[tid];
    const float ss = block_sum128(yv * yv, sm.red[2]);
    const float inv = 1.0f / sqrtf(ss * (1.0f / (float)SSM_D) + 1e-6f);
    const float zt = z_in[(size_t)b * INNER + (size_t)vh * SSM_D + tid];
    y_out[((size_t)b * vcount + vl) * SSM_D + tid] = ((yv * inv) * norm_w[tid]) * siluf_acc(zt);
    if (ok && lane == 0) bulk_wait_all();
}

cudaError_t launch_gdn_decode(dz_ctx* ctx, int layer, const GdnDecodeDesc& d, const float* qkv,
                              const float* alpha, const float* beta, const float* z, float* y,
                              cudaStream_t st, int* n_launch) {
    const LayerState& L = ctx->layers[layer];
    const int vc = ctx->cfg.v_head_count;
    cudaFuncSetAttribute(gdn_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(GdnSmem));
    gdn_decode_kernel<<<dim3(vc, d.B), 128, sizeof(GdnSmem), st>>>(d, ctx->cfg.v_head_begin, L.d_ssm, L.conv_w,
                                                                   L.ssm_a, L.dt_bias, L.norm_w, qkv, alpha, beta,
                                                                   z, y, vc, ctx->d_err);
    *n_launch += 1;
    return cudaGetLastError();
}

}  // namespace dz
