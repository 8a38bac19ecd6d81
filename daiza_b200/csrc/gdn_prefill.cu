// gdn_prefill.cu -- chunked (C = 64) Gated DeltaNet prefill on the tcgen05 tensor cores.
//
// Reference: Daiza-engine/src/model/forward.rs:897-1059 -- Phase A (conv1d from
// in-batch rows or pre-batch ring slots (h0+t+ct+1)%4, SiLU, L2-norm q/k,
// q *= 1/sqrt(128), silu(z)), the ring update (last min(4,T) rows, head =
// (h0+T)%4), and Phase B: per v head a chain over t of the fused row pass
// (model/ssm.rs:378-418) followed by the gated RMSNorm (ssm.rs:294-334).
//
// The token recurrence  S_t = e^{g_t} S_{t-1} + u_t k_t^T,
//                        u_t = beta_t (v_t - e^{g_t} S_{t-1} k_t),  y_t = S_t q_t
// (S stored [v][k]) is evaluated chunk by chunk in WY / UT form.  With G the
// in-chunk cumulative log decay, Gam_ts = e^{G_t - G_s},
// A = strict_lower(beta_t Gam_ts k_t.k_s) and Tm = (I + A)^-1:
//   U0 = Tm diag(beta) V,   W = Tm diag(beta e^G) K                  (per chunk)
//   U  = U0 - W S^T
//   Y  = diag(e^G) Q S^T + (lower_incl(Gam) o Q K^T) U
//   S' = e^{G_last} S + U^T diag(e^{G_last - G}) K                    (chunk to chunk)
// Every exponent is <= 0.
//
// Every matrix product runs on tcgen05 (kind::f16, f32 accumulation in TMEM)
// with both operands split into bf16 hi + lo halves and three products
// hi*hi + hi*lo + lo*hi, which keeps ~16 mantissa bits: the outputs and the
// final state stay ~1e-5 (relative, max-norm) from the f32 token recurrence.
//
// Kernels (stream-ordered):
//   gdn_pf_prep   per token: conv + SiLU + L2 norms + q scale + gates; writes
//                 q, k (every k head) and v (local v heads) as bf16 hi/lo rows
//                 [head][hi|lo][Tp][128] for TMA, log decay g and beta [head][Tp]
//   gdn_pf_ring   ring-buffer update (after every conv read)
//   gdn_pf_intra  one CTA per (chunk, v head): [K;Q] K^T, A and P, Tm by
//                 blocked forward substitution, W^T = K^T (Tm diag(beta e^G))^T
//                 and U0^T = V^T (Tm diag(beta))^T; writes an 80 KB record
//                 (W and P as ready-to-use operand images, U0^T, G)
//   gdn_pf_chain  one persistent CTA per v head: the state lives in TMEM as
//                 the f32 accumulator [128 v lanes][128 k columns] for the whole
//                 prefill; per chunk  U^T = U0^T - S W^T,  Y^T = S Qe^T + U^T P^T,
//                 S = e^{G_last} S + U^T Kd, with warp-specialised loader, MMA
//                 issuer and epilogues; the gated RMSNorm output is fused.
#include <cstddef>

#include "dz_internal.h"
#include "tc_common.cuh"

namespace dz {

namespace gp {
constexpr int C = 64;            // chunk length
constexpr int D = SSM_D;         // 128
// one (chunk, local v head) record written by gdn_pf_intra, read by gdn_pf_chain
constexpr uint32_t REC_W = 0;          // W  bf16 [hi|lo][k-box 2][64 t][64 k], K-major SW128 images (32 KB)
constexpr uint32_t REC_U0 = 32768;     // U0^T f32 [t-box 2][128 v][32 t], 16-byte chunks XOR-swizzled by v (32 KB)
constexpr uint32_t REC_P = 65536;      // P  bf16 [hi|lo][64 t][64 s], K-major SW128 images (16 KB)
constexpr uint32_t REC_G = 81920;      // G  f32 [64] in-chunk cumulative log decay
constexpr uint32_t REC_BYTES = 81920 + 256;
}  // namespace gp

// ---------------------------------------------------------------------------
// Phase A: conv1d + SiLU + L2 norms + gates, one CTA per (padded) token
// ---------------------------------------------------------------------------
__device__ __forceinline__ void store_split4(__nv_bfloat16* hi_row, size_t lo_offset, int lane, float4 x) {
    uint32_t h01, l01, h23, l23;
    tc::split2_bf16(x.x, x.y, h01, l01);
    tc::split2_bf16(x.z, x.w, h23, l23);
    *reinterpret_cast<uint2*>(hi_row + 4 * lane) = make_uint2(h01, h23);
    *reinterpret_cast<uint2*>(hi_row + lo_offset + 4 * lane) = make_uint2(l01, l23);
}

__global__ void __launch_bounds__(256) gdn_pf_prep_kernel(int64_t T, int64_t Tp, int vh0, int vc, int h0,
                                                          const float* __restrict__ qkv,
                                                          const float* __restrict__ hist,
                                                          const float* __restrict__ conv_w,
                                                          const float* __restrict__ ssm_a,
                                                          const float* __restrict__ dt_bias,
                                                          const float* __restrict__ alpha,
                                                          const float* __restrict__ beta,
                                                          __nv_bfloat16* __restrict__ qs, __nv_bfloat16* __restrict__ ks,
                                                          __nv_bfloat16* __restrict__ vs, float* __restrict__ gl,
                                                          float* __restrict__ bt) {
    const int64_t t = blockIdx.x;
    const bool pad = t >= T;     // rows of the last chunk past T: zero operands, g = 0, beta = 0
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const float qscale = 1.0f / sqrtf((float)SSM_D);
    const size_t lo_off = (size_t)Tp * SSM_D;
    for (int gi = warp; gi < 2 * SSM_HK + vc; gi += 8) {
        int cb;
        __nv_bfloat16* dst;
        if (gi < SSM_HK) {                              // q head
            cb = gi * SSM_D;
            dst = qs + ((size_t)gi * 2 * Tp + t) * SSM_D;
        } else if (gi < 2 * SSM_HK) {                   // k head
            cb = QKD + (gi - SSM_HK) * SSM_D;
            dst = ks + ((size_t)(gi - SSM_HK) * 2 * Tp + t) * SSM_D;
        } else {                                        // local v head
            cb = 2 * QKD + (vh0 + gi - 2 * SSM_HK) * SSM_D;
            dst = vs + ((size_t)(gi - 2 * SSM_HK) * 2 * Tp + t) * SSM_D;
        }
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        if (!pad) {
            const int ch = cb + 4 * lane;
#pragma unroll
            for (int ct = 0; ct < CONV_K; ++ct) {
                const int64_t st = t + ct - (CONV_K - 1);
                const float* src = st >= 0 ? qkv + st * QKV_LEN
                                           : hist + (size_t)((h0 + t + ct + 1) % CONV_K) * QKV_LEN;
                const float4 x = *reinterpret_cast<const float4*>(src + ch);
                const float4 w = *reinterpret_cast<const float4*>(conv_w + (size_t)ct * QKV_LEN + ch);
                acc.x = fmaf(x.x, w.x, acc.x);
                acc.y = fmaf(x.y, w.y, acc.y);
                acc.z = fmaf(x.z, w.z, acc.z);
                acc.w = fmaf(x.w, w.w, acc.w);
            }
            acc = make_float4(siluf_acc(acc.x), siluf_acc(acc.y), siluf_acc(acc.z), siluf_acc(acc.w));
            if (gi < 2 * SSM_HK) {
                const float ss = warp_sum(acc.x * acc.x + acc.y * acc.y + acc.z * acc.z + acc.w * acc.w);
                const float inv = 1.0f / sqrtf(ss + 1e-6f);
                acc = make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv);
                if (gi < SSM_HK) acc = make_float4(acc.x * qscale, acc.y * qscale, acc.z * qscale, acc.w * qscale);
            }
        }
        store_split4(dst, lo_off, lane, acc);
    }
    for (int vl = threadIdx.x; vl < vc; vl += blockDim.x) {
        const int vh = vh0 + vl;
        gl[(size_t)vl * Tp + t] = pad ? 0.0f : ssm_a[vh] * softplus_ref(alpha[(size_t)t * SSM_HV + vh] + dt_bias[vh]);
        bt[(size_t)vl * Tp + t] = pad ? 0.0f : sigmoidf_acc(beta[(size_t)t * SSM_HV + vh]);
    }
}

// ring update: the last m = min(4, T) raw rows land in slots (h0 + t) % 4
__global__ void gdn_pf_ring_kernel(int64_t T, int h0, const float* __restrict__ qkv, float* __restrict__ hist) {
    const int64_t m = T < CONV_K ? T : CONV_K;
    const int64_t t = T - m + blockIdx.x;
    const int slot = (int)((h0 + t) % CONV_K);
    for (int c = threadIdx.x; c < QKV_LEN / 4; c += blockDim.x)
        reinterpret_cast<float4*>(hist + (size_t)slot * QKV_LEN)[c] =
            reinterpret_cast<const float4*>(qkv + (size_t)t * QKV_LEN)[c];
}

template <typename S>
__device__ __forceinline__ S& align1024(unsigned char* raw) {
    return *reinterpret_cast<S*>((reinterpret_cast<uintptr_t>(raw) + 1023) & ~uintptr_t(1023));
}

// ---------------------------------------------------------------------------
// intra-chunk WY transform: one CTA (8 warps) per (chunk, local v head)
// ---------------------------------------------------------------------------
namespace gp {
constexpr int TP = C + 4;        // padded f32 row for the 64x64 triangular solve
struct alignas(1024) IntraSmem {
    // [hi|lo][d-box][row][64]: rows 0-63 = K of the chunk, 64-127 = Q.  After the
    // W / U0 products this 64 KB holds the W images (32 KB) then the U0^T image.
    __nv_bfloat16 kq[2][2][128][64];
    __nv_bfloat16 v[2][2][64][64];    // [hi|lo][d-box][s][64]
    __nv_bfloat16 tmw[2][64][64];     // Tm diag(beta e^G), [hi|lo][t][s] K-major
    __nv_bfloat16 tmb[2][64][64];     // Tm diag(beta)
    __nv_bfloat16 p[2][64][64];       // P image [hi|lo][t][s]
    float am[C][TP];                  // strictly lower beta_t Gam_ts k_t.k_s
    float tm[C][TP];                  // (I + A)^-1
    float g[C], b[C], G[C], eG[C];
    uint64_t bar_in, bar_m1, bar_m2;
    uint32_t tmem_base;
};
// TMEM columns of the intra kernel
constexpr uint32_t I_KQ = 0, I_W = 64, I_U0 = 128;
}  // namespace gp

__global__ void __launch_bounds__(256, 1) gdn_pf_intra_kernel(const __grid_constant__ CUtensorMap tm_q,
                                                              const __grid_constant__ CUtensorMap tm_k,
                                                              const __grid_constant__ CUtensorMap tm_v, int64_t Tp,
                                                              int vh0, int vc, const float* __restrict__ gl,
                                                              const float* __restrict__ bt,
                                                              unsigned char* __restrict__ rec, int* err) {
    using namespace gp;
    using namespace tc;
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    IntraSmem& sm = align1024<IntraSmem>(smem_raw);
    const int c = blockIdx.x, vl = blockIdx.y, tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31;
    const int kh = (vh0 + vl) % SSM_HK;
    const int t0 = c * C;

    if (warp == 0) tmem_alloc(&sm.tmem_base, 256);
    if (tid == 0) {
        mbar_init(&sm.bar_in, 1);
        mbar_init(&sm.bar_m1, 1);
        mbar_init(&sm.bar_m2, 1);
        fence_mbar_init();
    }
    fence_before_sync();
    __syncthreads();
    fence_after_sync();
    const uint32_t tmem = sm.tmem_base;
    bool ok = true;

    if (tid == 0) {
        mbar_arrive_expect_tx(&sm.bar_in, 12 * 8192 + 2 * 256);
        for (int hl = 0; hl < 2; ++hl)
            for (int db = 0; db < 2; ++db) {
                tma_load_4d(&sm.kq[hl][db][0][0], &tm_k, 64 * db, t0, hl, kh, &sm.bar_in);
                tma_load_4d(&sm.kq[hl][db][64][0], &tm_q, 64 * db, t0, hl, kh, &sm.bar_in);
                tma_load_4d(&sm.v[hl][db][0][0], &tm_v, 64 * db, t0, hl, vl, &sm.bar_in);
            }
        bulk_g2s(sm.g, gl + (size_t)vl * Tp + t0, 256, &sm.bar_in);
        bulk_g2s(sm.b, bt + (size_t)vl * Tp + t0, 256, &sm.bar_in);
    }
    wait_or_flag(&sm.bar_in, 0, err, ok);

    // ---- [K; Q] K^T  (M 128, N 64, K 128; three split products)
    if (tid == 0 && ok) {
        fence_after_sync();
        constexpr uint32_t ID = idesc_bf16(128, 64, false);
        const uint32_t kq_hi = smem_u32(&sm.kq[0][0][0][0]), kq_lo = smem_u32(&sm.kq[1][0][0][0]);
        uint32_t acc = 0;
        for (int pass = 0; pass < 3; ++pass) {
            const uint32_t a = pass == 2 ? kq_lo : kq_hi, b = pass == 1 ? kq_lo : kq_hi;
#pragma unroll
            for (int ks = 0; ks < 8; ++ks) {
                const uint32_t off = (uint32_t)(ks >> 2) * 16384u + (uint32_t)(ks & 3) * 32u;
                umma_ss(tmem + I_KQ, sw128_desc(a + off, 16, 1024), sw128_desc(b + off, 16, 1024), ID, acc);
                acc = 1;
            }
        }
        umma_commit(&sm.bar_m1);
    }
    if (warp == 1) {   // inclusive cumsum of the 64 log decays (2 per lane)
        const float a0 = sm.g[2 * lane], a1 = sm.g[2 * lane + 1];
        float s = a0 + a1;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const float y = __shfl_up_sync(0xffffffffu, s, o);
            if (lane >= o) s += y;
        }
        const float excl = s - (a0 + a1);
        sm.G[2 * lane] = excl + a0;
        sm.G[2 * lane + 1] = excl + a0 + a1;
        sm.eG[2 * lane] = expf(excl + a0);
        sm.eG[2 * lane + 1] = expf(excl + a0 + a1);
    }
    __syncthreads();

    // ---- epilogue 1: rows 0-63 -> A (f32, for the solve), rows 64-127 -> P image
    const int q4 = warp & 3, h = warp >> 2;
    const int row = 32 * q4 + lane;
    const uint32_t lane_addr = tmem + ((uint32_t)(32 * q4) << 16);
    if (wait_or_flag(&sm.bar_m1, 0, err, ok)) {
        fence_after_sync();
        float x[32];
        tmem_ld32(lane_addr + I_KQ + 32 * h, x);
        if (row < C) {
            const int t = row;
            const float bt_ = sm.b[t], Gt = sm.G[t];
#pragma unroll
            for (int j = 0; j < 32; ++j) {
                const int s = 32 * h + j;
                sm.am[t][s] = s < t ? bt_ * expf(Gt - sm.G[s]) * x[j] : 0.0f;
            }
        } else {
            const int t = row - C;
            const float Gt = sm.G[t];
#pragma unroll
            for (int j8 = 0; j8 < 4; ++j8) {
                uint4 hi, lo;
                uint32_t* hp = &hi.x;
                uint32_t* lp = &lo.x;
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int j = 8 * j8 + 2 * e, s = 32 * h + j;
                    const float p0 = s <= t ? expf(Gt - sm.G[s]) * x[j] : 0.0f;
                    const float p1 = s + 1 <= t ? expf(Gt - sm.G[s + 1]) * x[j + 1] : 0.0f;
                    split2_bf16(p0, p1, hp[e], lp[e]);
                }
                const uint32_t off = sw128_off_b16((uint32_t)t, (uint32_t)(32 * h + 8 * j8));
                *reinterpret_cast<uint4*>(reinterpret_cast<unsigned char*>(&sm.p[0][0][0]) + off) = hi;
                *reinterpret_cast<uint4*>(reinterpret_cast<unsigned char*>(&sm.p[1][0][0]) + off) = lo;
            }
        }
    }
    __syncthreads();

    // ---- Tm = (I + A)^-1, blocked 16x16.  Diagonal blocks: warp b, forward substitution.
    if (warp < 4) {
        const int b0 = 16 * warp;
        for (int i = 0; i < 16; ++i) {
            if (lane < 16) {
                const int j = lane;
                float xv = (i == j) ? 1.0f : 0.0f;
                for (int s = j; s < i; ++s) xv = fmaf(-sm.am[b0 + i][b0 + s], sm.tm[b0 + s][b0 + j], xv);
                sm.tm[b0 + i][b0 + j] = (j <= i) ? xv : 0.0f;
                for (int jj = b0 + 16; jj < C; jj += 16) sm.tm[b0 + i][jj + j] = 0.0f;   // strictly upper blocks
            }
            __syncwarp();
        }
    }
    __syncthreads();
    // off-diagonal blocks by block diagonal d: T_IJ = -T_II * sum_{K=J}^{I-1} A_IK T_KJ
    for (int d = 1; d < 4; ++d) {
        if (warp < 4 - d) {
            const int J = warp, I = warp + d;
            const int r = lane >> 1, cb = 8 * (lane & 1);
            float m[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) m[e] = 0.0f;
            for (int Kb = J; Kb < I; ++Kb)
                for (int s = 0; s < 16; ++s) {
                    const float a = sm.am[16 * I + r][16 * Kb + s];
#pragma unroll
                    for (int e = 0; e < 8; ++e) m[e] = fmaf(a, sm.tm[16 * Kb + s][16 * J + cb + e], m[e]);
                }
#pragma unroll
            for (int e = 0; e < 8; ++e) sm.tm[16 * I + r][16 * J + cb + e] = m[e];
            __syncwarp();
            float o[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) o[e] = 0.0f;
            for (int s = 0; s <= r; ++s) {
                const float tii = sm.tm[16 * I + r][16 * I + s];
#pragma unroll
                for (int e = 0; e < 8; ++e) o[e] = fmaf(tii, sm.tm[16 * I + s][16 * J + cb + e], o[e]);
            }
            __syncwarp();
#pragma unroll
            for (int e = 0; e < 8; ++e) sm.tm[16 * I + r][16 * J + cb + e] = -o[e];
        }
        __syncthreads();
    }
    // ---- Tm diag(beta e^G) and Tm diag(beta) as split K-major images [t][s]
    for (int i = tid; i < C * 8; i += 256) {
        const int t = i >> 3, j8 = i & 7;
        uint4 wh, wl, bh, bl;
        uint32_t *whp = &wh.x, *wlp = &wl.x, *bhp = &bh.x, *blp = &bl.x;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int s = 8 * j8 + 2 * e;
            const float a0 = sm.tm[t][s], a1 = sm.tm[t][s + 1];
            const float cb0 = sm.b[s], cb1 = sm.b[s + 1];
            split2_bf16(a0 * cb0 * sm.eG[s], a1 * cb1 * sm.eG[s + 1], whp[e], wlp[e]);
            split2_bf16(a0 * cb0, a1 * cb1, bhp[e], blp[e]);
        }
        const uint32_t off = sw128_off_b16((uint32_t)t, (uint32_t)(8 * j8));
        *reinterpret_cast<uint4*>(reinterpret_cast<unsigned char*>(&sm.tmw[0][0][0]) + off) = wh;
        *reinterpret_cast<uint4*>(reinterpret_cast<unsigned char*>(&sm.tmw[1][0][0]) + off) = wl;
        *reinterpret_cast<uint4*>(reinterpret_cast<unsigned char*>(&sm.tmb[0][0][0]) + off) = bh;
        *reinterpret_cast<uint4*>(reinterpret_cast<unsigned char*>(&sm.tmb[1][0][0]) + off) = bl;
    }
    fence_proxy_async_smem();
    __syncthreads();

    // ---- W^T = K^T TmW^T and U0^T = V^T TmB^T  (M 128 over k / v, N 64, K 64; A MN-major)
    if (tid == 0 && ok) {
        fence_after_sync();
        constexpr uint32_t ID = idesc_bf16(128, 64, false, true);
        const uint32_t k_hi = smem_u32(&sm.kq[0][0][0][0]), k_lo = smem_u32(&sm.kq[1][0][0][0]);
        const uint32_t v_hi = smem_u32(&sm.v[0][0][0][0]), v_lo = smem_u32(&sm.v[1][0][0][0]);
        const uint32_t w_hi = smem_u32(&sm.tmw[0][0][0]), w_lo = smem_u32(&sm.tmw[1][0][0]);
        const uint32_t b_hi = smem_u32(&sm.tmb[0][0][0]), b_lo = smem_u32(&sm.tmb[1][0][0]);
        uint32_t acc = 0;
        for (int pass = 0; pass < 3; ++pass) {
            const uint32_t a = pass == 2 ? k_lo : k_hi, b = pass == 1 ? w_lo : w_hi;
#pragma unroll
            for (int ks = 0; ks < 4; ++ks) {
                // A: K rows s (128 B of d each), d blocks of 64 in the 16 KB d-boxes
                umma_ss(tmem + I_W, sw128_desc(a + (uint32_t)ks * 2048u, 16384, 1024),
                        sw128_desc(b + (uint32_t)ks * 32u, 16, 1024), ID, acc);
                acc = 1;
            }
        }
        acc = 0;
        for (int pass = 0; pass < 3; ++pass) {
            const uint32_t a = pass == 2 ? v_lo : v_hi, b = pass == 1 ? b_lo : b_hi;
#pragma unroll
            for (int ks = 0; ks < 4; ++ks) {
                umma_ss(tmem + I_U0, sw128_desc(a + (uint32_t)ks * 2048u, 8192, 1024),
                        sw128_desc(b + (uint32_t)ks * 32u, 16, 1024), ID, acc);
                acc = 1;
            }
        }
        umma_commit(&sm.bar_m2);
    }
    unsigned char* img = reinterpret_cast<unsigned char*>(&sm.kq[0][0][0][0]);   // W images, then U0^T image
    if (wait_or_flag(&sm.bar_m2, 0, err, ok)) {
        fence_after_sync();
        float x[32];
        // W^T: lane = k, columns t in [32h, 32h + 32) -> W[t][k] images
        tmem_ld32(lane_addr + I_W + 32 * h, x);
        {
            const uint32_t kb = (uint32_t)row >> 6, kc = (uint32_t)row & 63u;
#pragma unroll
            for (int j = 0; j < 32; ++j) {
                __nv_bfloat16 hi, lo;
                split_bf16(x[j], hi, lo);
                const uint32_t off = kb * 8192u + sw128_off_b16((uint32_t)(32 * h + j), kc);
                *reinterpret_cast<__nv_bfloat16*>(img + off) = hi;
                *reinterpret_cast<__nv_bfloat16*>(img + 16384 + off) = lo;
            }
        }
        // U0^T: lane = v, columns t in [32h, 32h + 32) -> t-box h of the f32 image
        tmem_ld32(lane_addr + I_U0 + 32 * h, x);
#pragma unroll
        for (int j4 = 0; j4 < 8; ++j4)
            *reinterpret_cast<float4*>(img + REC_U0 + (uint32_t)h * 16384u + sw128_off_b32((uint32_t)row, 4u * j4)) =
                make_float4(x[4 * j4], x[4 * j4 + 1], x[4 * j4 + 2], x[4 * j4 + 3]);
    }
    fence_proxy_async_smem();
    __syncthreads();
    if (tid == 0 && ok) {
        unsigned char* R = rec + ((size_t)c * vc + vl) * REC_BYTES;
        bulk_s2g(R + REC_W, img, 65536);
        bulk_s2g(R + REC_P, &sm.p[0][0][0], 16384);
        bulk_s2g(R + REC_G, sm.G, 256);
        bulk_commit();
        bulk_wait_all();
    }
    fence_before_sync();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tmem, 256);
}

// ---------------------------------------------------------------------------
// chunk recurrence: one persistent CTA per local v head
// ---------------------------------------------------------------------------
namespace gp {
struct alignas(1024) ChainSmem {
    unsigned char w[32768];      // record: W images [hi|lo][k-box][64 t][64 k]
    unsigned char u0t[32768];    // record: U0^T image [t-box][128 v][32 t]
    unsigned char p[16384];      // record: P images [hi|lo][64 t][64 s]
    unsigned char qe[32768];     // Q [hi|lo][d-box][64 t][64 d] as loaded, scaled in place to Q e^G
    unsigned char kd[32768];     // K e^{G_last - G}, same layout (B operand, MN-major)
    unsigned char kraw[32768];   // K as loaded
    float zt[C][D];              // z rows of the chunk for this head [t][v] (TMA, zero past T)
    float gring[4][C];           // G of chunks c % 4
    float red[4][C];             // per-warp partial sums of y^2 per token
    float inv[C];                // 1 / rms per token
    uint64_t full_w, full_u0, full_p, full_q, full_k, full_z, full_g[4];
    uint64_t mma1_done, dy1_done, mma3_done;
    uint64_t mma2_done[2], y_free[2];   // per D_Y buffer (chunk parity): one completion every 2 chunks
    uint64_t s_ready, u_ready, qe_ready, kd_ready, z_free;
    uint32_t tmem_base;
};
// TMEM columns of the chain kernel (512 allocated)
constexpr uint32_t S_ACC = 0;    // f32 state [v lane][k], holds e^{G_last} S between the S epilogue and MMA3
constexpr uint32_t S_HI = 128;   // bf16 pairs of S (A operand), 64 columns
constexpr uint32_t S_LO = 192;
constexpr uint32_t D_U = 256;    // S W^T, f32 [v][t]
constexpr uint32_t U_HI = 320;   // bf16 pairs of U^T (A operand), 32 columns
constexpr uint32_t U_LO = 352;
constexpr uint32_t D_Y = 384;    // Y^T f32 [v][t], two buffers (chunk parity) at 384 and 448
// warp roles
constexpr int EY_W0 = 0;         // warps 0-3: y epilogue (gated RMSNorm, store)
constexpr int E1_W0 = 4;         // warps 4-11: U and S epilogues (the serial path)
constexpr int ES_W0 = 12;        // warps 12-15: Q e^G and K e^{G_last - G} scaling
constexpr int CTL_W = 16;        // warp 16: lane 0 loads, lane 1 issues MMAs
constexpr int CHAIN_THREADS = 17 * 32;
}  // namespace gp

__device__ __forceinline__ bool named_bar_and(int id, int nthreads, bool pred) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\t"
        "barrier.red.and.pred q, %2, %3, p;\n\tselp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(r) : "r"((uint32_t)pred), "r"(id), "r"(nthreads) : "memory");
    return r != 0;
}

// One halving step of a warp reduce-scatter: N values per lane -> N/2, lanes
// with BIT set keep (and sum) the upper half.
template <int N, int BIT>
__device__ __forceinline__ void bfly_reduce(float* a, int lane) {
    const bool up = (lane & BIT) != 0;
#pragma unroll
    for (int j = 0; j < N / 2; ++j) {
        const float keep = up ? a[j + N / 2] : a[j];
        const float send = up ? a[j] : a[j + N / 2];
        a[j] = keep + __shfl_xor_sync(0xffffffffu, send, BIT);
    }
}

// scale each 128-byte row t of a [hi|lo][d-box][64][64] bf16 image by f(t), re-splitting hi/lo
template <typename F>
__device__ __forceinline__ void scale_rows(const unsigned char* src, unsigned char* dst, int tid, int nthr, F f) {
    for (int i = tid; i < 1024; i += nthr) {          // 16-byte chunks of the hi image
        const uint32_t off = (uint32_t)i * 16u;
        const int t = (int)((off & 8191u) >> 7);
        const float sc = f(t);
        const uint4 h = *reinterpret_cast<const uint4*>(src + off);
        const uint4 l = *reinterpret_cast<const uint4*>(src + 16384 + off);
        const uint32_t* hp = &h.x;
        const uint32_t* lp = &l.x;
        uint4 nh, nl;
        uint32_t* nhp = &nh.x;
        uint32_t* nlp = &nl.x;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const float a = (tc::bf16_lo_f(hp[e]) + tc::bf16_lo_f(lp[e])) * sc;
            const float b = (tc::bf16_hi_f(hp[e]) + tc::bf16_hi_f(lp[e])) * sc;
            tc::split2_bf16(a, b, nhp[e], nlp[e]);
        }
        *reinterpret_cast<uint4*>(dst + off) = nh;
        *reinterpret_cast<uint4*>(dst + 16384 + off) = nl;
    }
}

__global__ void __launch_bounds__(gp::CHAIN_THREADS, 1) gdn_pf_chain_kernel(
    const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
    const __grid_constant__ CUtensorMap tm_z, int64_t T, int NC, int vh0, int vc, const unsigned char* __restrict__ rec,
    float* __restrict__ state, const float* __restrict__ norm_w, float* __restrict__ y_out, int* err) {
    using namespace gp;
    using namespace tc;
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    ChainSmem& sm = align1024<ChainSmem>(smem_raw);
    const int vl = blockIdx.x, tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31;
    const int kh = (vh0 + vl) % SSM_HK;
    auto R = [&](int c) { return rec + ((size_t)c * vc + vl) * REC_BYTES; };

    if (warp == CTL_W) tmem_alloc(&sm.tmem_base, 512);
    if (tid == 0) {
        uint64_t* one[11] = {&sm.full_w, &sm.full_u0, &sm.full_p, &sm.full_q, &sm.full_k, &sm.full_z,
                             &sm.mma1_done, &sm.dy1_done, &sm.mma3_done, &sm.mma2_done[0], &sm.mma2_done[1]};
        for (uint64_t* b : one) mbar_init(b, 1);
        for (int i = 0; i < 4; ++i) mbar_init(&sm.full_g[i], 1);
        mbar_init(&sm.s_ready, 256);
        mbar_init(&sm.u_ready, 256);
        mbar_init(&sm.qe_ready, 128);
        mbar_init(&sm.kd_ready, 128);
        mbar_init(&sm.y_free[0], 128);
        mbar_init(&sm.y_free[1], 128);
        mbar_init(&sm.z_free, 128);
        fence_mbar_init();
    }
    fence_before_sync();
    __syncthreads();
    fence_after_sync();
    const uint32_t tmem = sm.tmem_base;
    bool ok = true;

    if (warp == CTL_W) {
        if (lane == 0) {
            // ---------------- loader ----------------
            for (int c = 0; c < NC && c < 3; ++c) {
                mbar_arrive_expect_tx(&sm.full_g[c], 256);
                bulk_g2s(sm.gring[c], R(c) + REC_G, 256, &sm.full_g[c]);
            }
            for (int c = 0; c < NC && ok; ++c) {
                const uint32_t pp = (uint32_t)((c - 1) & 1);
                const int t0 = c * C;
                if (c > 0 && !wait_or_flag(&sm.kd_ready, pp, err, ok)) break;
                mbar_arrive_expect_tx(&sm.full_k, 32768);
                for (int hl = 0; hl < 2; ++hl)
                    for (int db = 0; db < 2; ++db)
                        tma_load_4d(sm.kraw + hl * 16384 + db * 8192, &tm_k, 64 * db, t0, hl, kh, &sm.full_k);
                if (c > 0 && !wait_or_flag(&sm.mma1_done, pp, err, ok)) break;
                mbar_arrive_expect_tx(&sm.full_w, 32768);
                bulk_g2s(sm.w, R(c) + REC_W, 32768, &sm.full_w);
                if (c > 0 && !wait_or_flag(&sm.u_ready, pp, err, ok)) break;
                mbar_arrive_expect_tx(&sm.full_u0, 32768);
                bulk_g2s(sm.u0t, R(c) + REC_U0, 32768, &sm.full_u0);
                if (c > 0 && !wait_or_flag(&sm.dy1_done, pp, err, ok)) break;
                mbar_arrive_expect_tx(&sm.full_q, 32768);
                for (int hl = 0; hl < 2; ++hl)
                    for (int db = 0; db < 2; ++db)
                        tma_load_4d(sm.qe + hl * 16384 + db * 8192, &tm_q, 64 * db, t0, hl, kh, &sm.full_q);
                if (c > 0 && !wait_or_flag(&sm.mma2_done[(c - 1) & 1], (uint32_t)(((c - 1) >> 1) & 1), err, ok)) break;
                mbar_arrive_expect_tx(&sm.full_p, 16384);
                bulk_g2s(sm.p, R(c) + REC_P, 16384, &sm.full_p);
                if (c > 0 && !wait_or_flag(&sm.z_free, pp, err, ok)) break;
                mbar_arrive_expect_tx(&sm.full_z, C * D * 4);
                tma_load_2d(&sm.zt[0][0], &tm_z, (vh0 + vl) * D, t0, &sm.full_z);
                // G of chunk c+3 into slot (c+3)%4 (chunk c-1's G: every reader finished before MMA2(c-1))
                if (c + 3 < NC) {
                    const int s = (c + 3) & 3;
                    mbar_arrive_expect_tx(&sm.full_g[s], 256);
                    bulk_g2s(sm.gring[s], R(c + 3) + REC_G, 256, &sm.full_g[s]);
                }
            }
        } else if (lane == 1) {
            // ---------------- MMA issuer ----------------
            constexpr uint32_t ID64 = idesc_bf16(128, 64, false);
            constexpr uint32_t ID128MN = idesc_bf16(128, 128, true);
            const uint32_t w_s = smem_u32(sm.w), q_s = smem_u32(sm.qe), k_s = smem_u32(sm.kd), p_s = smem_u32(sm.p);
            for (int c = 0; c < NC && ok; ++c) {
                const uint32_t ph = (uint32_t)(c & 1);
                // U-part: D_U = S W^T  (A = S hi/lo from TMEM, B = W images, N 64, K 128)
                if (!wait_or_flag(&sm.s_ready, ph, err, ok) || !wait_or_flag(&sm.full_w, ph, err, ok)) break;
                fence_after_sync();
                {
                    uint32_t acc = 0;
                    for (int pass = 0; pass < 3; ++pass) {
                        const uint32_t a = pass == 2 ? S_LO : S_HI, b = w_s + (pass == 1 ? 16384u : 0u);
#pragma unroll
                        for (int ks = 0; ks < 8; ++ks) {
                            umma_ts(tmem + D_U, tmem + a + 8u * ks,
                                    sw128_desc(b + (uint32_t)(ks >> 2) * 8192u + (uint32_t)(ks & 3) * 32u, 16, 1024),
                                    ID64, acc);
                            acc = 1;
                        }
                    }
                }
                umma_commit(&sm.mma1_done);
                // Y-part 1: D_Y = S Qe^T
                if (!wait_or_flag(&sm.qe_ready, ph, err, ok)) break;
                if (c > 1 && !wait_or_flag(&sm.y_free[c & 1], (uint32_t)(((c - 2) >> 1) & 1), err, ok)) break;
                const uint32_t dy = D_Y + 64u * (uint32_t)(c & 1);
                fence_after_sync();
                {
                    uint32_t acc = 0;
                    for (int pass = 0; pass < 3; ++pass) {
                        const uint32_t a = pass == 2 ? S_LO : S_HI, b = q_s + (pass == 1 ? 16384u : 0u);
#pragma unroll
                        for (int ks = 0; ks < 8; ++ks) {
                            umma_ts(tmem + dy, tmem + a + 8u * ks,
                                    sw128_desc(b + (uint32_t)(ks >> 2) * 8192u + (uint32_t)(ks & 3) * 32u, 16, 1024),
                                    ID64, acc);
                            acc = 1;
                        }
                    }
                }
                umma_commit(&sm.dy1_done);
                // state: S_ACC (= e^{G_last} S) += U^T Kd  (B = Kd MN-major, N 128, K 64)
                if (!wait_or_flag(&sm.u_ready, ph, err, ok) || !wait_or_flag(&sm.kd_ready, ph, err, ok)) break;
                fence_after_sync();
                for (int pass = 0; pass < 3; ++pass) {
                    const uint32_t a = pass == 2 ? U_LO : U_HI, b = k_s + (pass == 1 ? 16384u : 0u);
#pragma unroll
                    for (int ks = 0; ks < 4; ++ks)
                        umma_ts(tmem + S_ACC, tmem + a + 8u * ks, sw128_desc(b + (uint32_t)ks * 2048u, 8192, 1024),
                                ID128MN, 1);
                }
                umma_commit(&sm.mma3_done);
                // Y-part 2: D_Y += U^T P^T  (B = P images, N 64, K 64)
                if (!wait_or_flag(&sm.full_p, ph, err, ok)) break;
                fence_after_sync();
                for (int pass = 0; pass < 3; ++pass) {
                    const uint32_t a = pass == 2 ? U_LO : U_HI, b = p_s + (pass == 1 ? 8192u : 0u);
#pragma unroll
                    for (int ks = 0; ks < 4; ++ks)
                        umma_ts(tmem + dy, tmem + a + 8u * ks, sw128_desc(b + (uint32_t)ks * 32u, 16, 1024), ID64, 1);
                }
                umma_commit(&sm.mma2_done[c & 1]);
            }
        }
    } else if (warp >= E1_W0 && warp < ES_W0) {
        // ---------------- U and S epilogues (thread = state row v, half h of the columns) ----------------
        const int q4 = warp & 3, h = (warp - E1_W0) >> 2;
        const int v = 32 * q4 + lane;
        const uint32_t la = tmem + ((uint32_t)(32 * q4) << 16);
        float* Sg = state + ((size_t)vl * D + v) * D;
        // initial state: S_HI/S_LO <- split(S0), S_ACC <- e^{G_last(0)} S0
        if (wait_or_flag(&sm.full_g[0], 0, err, ok)) {
            const float e0 = expf(sm.gring[0][C - 1]);
            for (int piece = 0; piece < 2; ++piece) {
                const int k0 = 64 * h + 32 * piece;
                uint32_t hi[16], lo[16], sc[32];
#pragma unroll
                for (int j4 = 0; j4 < 8; ++j4) {
                    const float4 s4 = *reinterpret_cast<const float4*>(Sg + k0 + 4 * j4);
                    split2_bf16(s4.x, s4.y, hi[2 * j4], lo[2 * j4]);
                    split2_bf16(s4.z, s4.w, hi[2 * j4 + 1], lo[2 * j4 + 1]);
                    sc[4 * j4] = __float_as_uint(s4.x * e0);
                    sc[4 * j4 + 1] = __float_as_uint(s4.y * e0);
                    sc[4 * j4 + 2] = __float_as_uint(s4.z * e0);
                    sc[4 * j4 + 3] = __float_as_uint(s4.w * e0);
                }
                tmem_st16_async(la + S_HI + (uint32_t)(k0 >> 1), hi);
                tmem_st16_async(la + S_LO + (uint32_t)(k0 >> 1), lo);
                tmem_st32_async(la + S_ACC + (uint32_t)k0, sc);
            }
            tmem_wait_st();
        }
        fence_before_sync();
        mbar_arrive(&sm.s_ready);
        for (int c = 0; c < NC && ok; ++c) {
            const uint32_t ph = (uint32_t)(c & 1);
            // U^T = U0^T - S W^T  -> bf16 pairs (columns t in [32h, 32h + 32))
            if (!wait_or_flag(&sm.mma1_done, ph, err, ok) || !wait_or_flag(&sm.full_u0, ph, err, ok)) break;
            fence_after_sync();
            {
                float x[32];
                tmem_ld32(la + D_U + 32u * h, x);
                uint32_t hi[16], lo[16];
                const unsigned char* u0 = sm.u0t + (uint32_t)h * 16384u;
#pragma unroll
                for (int j4 = 0; j4 < 8; ++j4) {
                    const float4 a = *reinterpret_cast<const float4*>(u0 + sw128_off_b32((uint32_t)v, 4u * j4));
                    split2_bf16(a.x - x[4 * j4], a.y - x[4 * j4 + 1], hi[2 * j4], lo[2 * j4]);
                    split2_bf16(a.z - x[4 * j4 + 2], a.w - x[4 * j4 + 3], hi[2 * j4 + 1], lo[2 * j4 + 1]);
                }
                tmem_st16_async(la + U_HI + 16u * h, hi);
                tmem_st16_async(la + U_LO + 16u * h, lo);
                tmem_wait_st();
            }
            fence_before_sync();
            mbar_arrive(&sm.u_ready);
            // S epilogue: S_{c+1} -> S_HI/S_LO and S_ACC <- e^{G_last(c+1)} S_{c+1}; or the final state
            if (!wait_or_flag(&sm.mma3_done, ph, err, ok)) break;
            fence_after_sync();
            const bool last = c + 1 == NC;
            float e1 = 1.0f;
            if (!last) {
                const int s = (c + 1) & 3;
                if (!wait_or_flag(&sm.full_g[s], (uint32_t)(((c + 1) >> 2) & 1), err, ok)) break;
                e1 = expf(sm.gring[s][C - 1]);
            }
            for (int piece = 0; piece < 2; ++piece) {
                const int k0 = 64 * h + 32 * piece;
                uint32_t r[32];
                tmem_ld32_async(la + S_ACC + (uint32_t)k0, r);
                tmem_wait_ld();
                if (last) {
#pragma unroll
                    for (int j4 = 0; j4 < 8; ++j4)
                        *reinterpret_cast<float4*>(Sg + k0 + 4 * j4) =
                            make_float4(__uint_as_float(r[4 * j4]), __uint_as_float(r[4 * j4 + 1]),
                                        __uint_as_float(r[4 * j4 + 2]), __uint_as_float(r[4 * j4 + 3]));
                } else {
                    uint32_t hi[16], lo[16];
#pragma unroll
                    for (int j = 0; j < 16; ++j)
                        split2_bf16(__uint_as_float(r[2 * j]), __uint_as_float(r[2 * j + 1]), hi[j], lo[j]);
                    tmem_st16_async(la + S_HI + (uint32_t)(k0 >> 1), hi);
                    tmem_st16_async(la + S_LO + (uint32_t)(k0 >> 1), lo);
#pragma unroll
                    for (int j = 0; j < 32; ++j) r[j] = __float_as_uint(__uint_as_float(r[j]) * e1);
                    tmem_st32_async(la + S_ACC + (uint32_t)k0, r);
                }
            }
            if (!last) {
                tmem_wait_st();
                fence_before_sync();
                mbar_arrive(&sm.s_ready);
            }
        }
    } else if (warp >= ES_W0) {
        // ---------------- Q e^G and K e^{G_last - G} ----------------
        const int et = tid - ES_W0 * 32;
        for (int c = 0; c < NC && ok; ++c) {
            const uint32_t ph = (uint32_t)(c & 1);
            const int s = c & 3;
            if (!wait_or_flag(&sm.full_g[s], (uint32_t)((c >> 2) & 1), err, ok)) break;
            const float* G = sm.gring[s];
            if (!wait_or_flag(&sm.full_q, ph, err, ok)) break;
            scale_rows(sm.qe, sm.qe, et, 128, [&](int t) { return expf(G[t]); });
            fence_proxy_async_smem();
            mbar_arrive(&sm.qe_ready);
            if (!wait_or_flag(&sm.full_k, ph, err, ok)) break;
            if (c > 0 && !wait_or_flag(&sm.mma3_done, (uint32_t)((c - 1) & 1), err, ok)) break;
            const float Gl = G[C - 1];
            scale_rows(sm.kraw, sm.kd, et, 128, [&](int t) { return expf(Gl - G[t]); });
            fence_proxy_async_smem();
            mbar_arrive(&sm.kd_ready);
        }
    } else {
        // ---------------- y epilogue: gated RMSNorm of Y^T, thread = v ----------------
        const int ew = warp - EY_W0;
        const int v = 32 * ew + lane;
        const uint32_t la = tmem + ((uint32_t)(32 * ew) << 16);
        const float wv = norm_w[v];
        float* yb = y_out + (size_t)vl * D + v;
        for (int c = 0; c < NC; ++c) {
            const bool got = ok && wait_or_flag(&sm.mma2_done[c & 1], (uint32_t)((c >> 1) & 1), err, ok);
            if (!named_bar_and(1, 128, got)) {
                ok = false;
                break;
            }
            fence_after_sync();
            float y[C];
            {
                uint32_t r[32];
                const uint32_t dy = D_Y + 64u * (uint32_t)(c & 1);
                tmem_ld32_async(la + dy, r);
                tmem_wait_ld();
#pragma unroll
                for (int j = 0; j < 32; ++j) y[j] = __uint_as_float(r[j]);
                tmem_ld32_async(la + dy + 32u, r);
                tmem_wait_ld();
#pragma unroll
                for (int j = 0; j < 32; ++j) y[32 + j] = __uint_as_float(r[j]);
            }
            fence_before_sync();
            mbar_arrive(&sm.y_free[c & 1]);
            // sum over this warp's 32 v of y^2 for each of the 64 tokens: halving butterfly,
            // lane L ends with tokens 2L and 2L+1
            float a[C];
#pragma unroll
            for (int j = 0; j < C; ++j) a[j] = y[j] * y[j];
            bfly_reduce<64, 16>(a, lane);
            bfly_reduce<32, 8>(a, lane);
            bfly_reduce<16, 4>(a, lane);
            bfly_reduce<8, 2>(a, lane);
            bfly_reduce<4, 1>(a, lane);
            sm.red[ew][2 * lane] = a[0];
            sm.red[ew][2 * lane + 1] = a[1];
            tc::named_bar_sync(1, 128);
            if (ew < 2) {
                const int t = 32 * ew + lane;
                const float ss = (sm.red[0][t] + sm.red[1][t]) + (sm.red[2][t] + sm.red[3][t]);
                sm.inv[t] = 1.0f / sqrtf(ss / (float)D + 1e-6f);
            }
            tc::named_bar_sync(1, 128);
            const bool zok = wait_or_flag(&sm.full_z, (uint32_t)(c & 1), err, ok);
            const int64_t t0 = (int64_t)c * C;
            const int n = (int)(T - t0 < C ? T - t0 : C);
            if (zok) {
#pragma unroll
                for (int t = 0; t < C; ++t)
                    if (t < n)
                        yb[(size_t)(t0 + t) * vc * D] = ((y[t] * sm.inv[t]) * wv) * siluf_acc(sm.zt[t][v]);
            }
            mbar_arrive(&sm.z_free);
        }
    }
    fence_before_sync();
    __syncthreads();
    if (warp == CTL_W) tmem_dealloc(tmem, 512);
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
namespace {
// bf16 [heads][2][Tp][128] (hi | lo rows) with (64 x 64 x 1 x 1) boxes, 128-byte swizzle
bool make_split_map(CUtensorMap* m, const void* base, int64_t Tp, int heads) {
    EncodeTiledFn fn = tensor_map_encoder();
    if (!fn) return false;
    cuuint64_t dims[4] = {(cuuint64_t)SSM_D, (cuuint64_t)Tp, 2, (cuuint64_t)heads};
    cuuint64_t strides[3] = {(cuuint64_t)SSM_D * 2, (cuuint64_t)Tp * SSM_D * 2, (cuuint64_t)2 * Tp * SSM_D * 2};
    cuuint32_t box[4] = {64, 64, 1, 1};
    cuuint32_t estr[4] = {1, 1, 1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}
// z [T][6144] f32 with (128 x 64) boxes, no swizzle; rows past T read as zero
bool make_z_map(CUtensorMap* m, const float* z, int64_t T) {
    EncodeTiledFn fn = tensor_map_encoder();
    if (!fn) return false;
    cuuint64_t dims[2] = {(cuuint64_t)INNER, (cuuint64_t)T};
    cuuint64_t strides[1] = {(cuuint64_t)INNER * 4};
    cuuint32_t box[2] = {(cuuint32_t)SSM_D, (cuuint32_t)gp::C};
    cuuint32_t estr[2] = {1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(z), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}
size_t round_up(size_t x, size_t a) { return (x + a - 1) / a * a; }
}  // namespace

cudaError_t launch_gdn_prefill(dz_ctx* ctx, int layer, int seq, int64_t T, const float* qkv, const float* alpha,
                               const float* beta, const float* z, float* y, cudaStream_t st, int* n_launch) {
    using namespace gp;
    const LayerState& L = ctx->layers[layer];
    const int vh0 = ctx->cfg.v_head_begin, vc = ctx->cfg.v_head_count;
    const SsmSlot slot = L.h_ssm[seq];
    const int h0 = L.head[seq];
    const int NC = (int)((T + C - 1) / C);
    const int64_t Tp = (int64_t)NC * C;
    // scratch: q/k/v operand rows, gates, records
    const size_t qk_bytes = round_up((size_t)SSM_HK * 2 * Tp * D * 2, 1024);
    const size_t v_bytes = round_up((size_t)vc * 2 * Tp * D * 2, 1024);
    const size_t g_bytes = round_up((size_t)vc * Tp * 4, 1024);
    const size_t rec_bytes = (size_t)NC * vc * REC_BYTES;
    cudaError_t e = ensure_prefill_scratch(ctx, 2 * qk_bytes + v_bytes + 2 * g_bytes + rec_bytes + 1024);
    if (e != cudaSuccess) return e;
    unsigned char* base = reinterpret_cast<unsigned char*>(round_up(reinterpret_cast<uintptr_t>(ctx->pf), 1024));
    __nv_bfloat16* qs = reinterpret_cast<__nv_bfloat16*>(base);
    __nv_bfloat16* ks = reinterpret_cast<__nv_bfloat16*>(base + qk_bytes);
    __nv_bfloat16* vs = reinterpret_cast<__nv_bfloat16*>(base + 2 * qk_bytes);
    float* gl = reinterpret_cast<float*>(base + 2 * qk_bytes + v_bytes);
    float* bt = reinterpret_cast<float*>(base + 2 * qk_bytes + v_bytes + g_bytes);
    unsigned char* rec = base + 2 * qk_bytes + v_bytes + 2 * g_bytes;

    CUtensorMap mq, mk, mv, mz;
    if (!make_split_map(&mq, qs, Tp, SSM_HK) || !make_split_map(&mk, ks, Tp, SSM_HK) ||
        !make_split_map(&mv, vs, Tp, vc) || !make_z_map(&mz, z, T))
        return cudaErrorInvalidValue;

    gdn_pf_prep_kernel<<<(unsigned)Tp, 256, 0, st>>>(T, Tp, vh0, vc, h0, qkv, slot.hist, L.conv_w, L.ssm_a,
                                                     L.dt_bias, alpha, beta, qs, ks, vs, gl, bt);
    gdn_pf_ring_kernel<<<(unsigned)(T < CONV_K ? T : CONV_K), 256, 0, st>>>(T, h0, qkv, slot.hist);
    const int smem_i = (int)sizeof(IntraSmem) + 1024;
    e = cudaFuncSetAttribute(gdn_pf_intra_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_i);
    if (e != cudaSuccess) return e;
    gdn_pf_intra_kernel<<<dim3(NC, vc), 256, smem_i, st>>>(mq, mk, mv, Tp, vh0, vc, gl, bt, rec, ctx->d_err);
    const int smem_c = (int)sizeof(ChainSmem) + 1024;
    e = cudaFuncSetAttribute(gdn_pf_chain_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_c);
    if (e != cudaSuccess) return e;
    gdn_pf_chain_kernel<<<vc, CHAIN_THREADS, smem_c, st>>>(mq, mk, mz, T, NC, vh0, vc, rec, slot.state, L.norm_w, y,
                                                           ctx->d_err);
    *n_launch += 4;
    return cudaGetLastError();
}

}  // namespace dz
