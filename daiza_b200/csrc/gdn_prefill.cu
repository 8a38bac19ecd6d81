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
//   gdn_pf_intra  persistent CTAs over the (chunk, v head) items: [K;Q] K^T,
//                 A and P, Tm by blocked forward substitution,
//                 W^T = K^T (Tm diag(beta e^G))^T and U0^T = V^T (Tm diag(beta))^T;
//                 writes an 80 KB record per item (W and P as ready-to-use
//                 operand images, U0^T, G)
//   gdn_pf_chain  one CTA per v head over a range of chunks: the state lives in
//                 TMEM as the f32 accumulator [128 v lanes][128 k columns]
//                 (loaded from and stored back to the SSM state at the ends of
//                 the range); per chunk  U^T = U0^T - S W^T,
//                 Y^T = S Qe^T + U^T P^T,  S = e^{G_last} S + U^T Kd, with
//                 warp-specialised loader, MMA issuer and epilogues; the gated
//                 RMSNorm output is fused.
// From 16 chunks on, the chunks are cut into segments: the intra kernel of
// segment k + 1 runs on a side stream (n_sm - vc CTAs) while the chain kernel of
// segment k runs on the caller's stream (vc CTAs); events order them, no kernel
// waits on another.
#include <algorithm>
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
// Phase A: conv1d + SiLU + L2 norms + gates, one CTA per 4 (padded) tokens
// ---------------------------------------------------------------------------
__device__ __forceinline__ void store_split4(__nv_bfloat16* hi_row, size_t lo_offset, int lane, float4 x) {
    uint32_t h01, l01, h23, l23;
    tc::split2_bf16(x.x, x.y, h01, l01);
    tc::split2_bf16(x.z, x.w, h23, l23);
    *reinterpret_cast<uint2*>(hi_row + 4 * lane) = make_uint2(h01, h23);
    *reinterpret_cast<uint2*>(hi_row + lo_offset + 4 * lane) = make_uint2(l01, l23);
}

constexpr int PREP_TOK = 4;      // tokens per prep CTA: conv weights and shared input rows are read once for 4 tokens

// silu with the fast exponential and division (relative error ~1e-6, far below
// the bf16 hi/lo operand split that follows)
__device__ __forceinline__ float silu_fast(float x) { return __fdividef(x, 1.0f + __expf(-x)); }

__global__ void __launch_bounds__(256, 4) gdn_pf_prep_kernel(int64_t T, int64_t Tp, int vh0, int vc, int h0,
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
    const int64_t tb = (int64_t)blockIdx.x * PREP_TOK;   // first token of this CTA (Tp is a multiple of 4)
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const float qscale = 1.0f / sqrtf((float)SSM_D);
    const size_t lo_off = (size_t)Tp * SSM_D;
    for (int gi = warp; gi < 2 * SSM_HK + vc; gi += 8) {
        int cb;
        __nv_bfloat16* dst;
        if (gi < SSM_HK) {                              // q head
            cb = gi * SSM_D;
            dst = qs + ((size_t)gi * 2 * Tp + tb) * SSM_D;
        } else if (gi < 2 * SSM_HK) {                   // k head
            cb = QKD + (gi - SSM_HK) * SSM_D;
            dst = ks + ((size_t)(gi - SSM_HK) * 2 * Tp + tb) * SSM_D;
        } else {                                        // local v head
            cb = 2 * QKD + (vh0 + gi - 2 * SSM_HK) * SSM_D;
            dst = vs + ((size_t)(gi - 2 * SSM_HK) * 2 * Tp + tb) * SSM_D;
        }
        const int ch = cb + 4 * lane;
        // input rows tb-3 .. tb+3 (ring slots (h0+t+ct+1)%4 before the batch; the reference's
        // tap order: t=0 oldest ... t=3 the token itself), weights of the 4 taps
        float4 x[PREP_TOK + CONV_K - 1], w[CONV_K];
#pragma unroll
        for (int ct = 0; ct < CONV_K; ++ct) w[ct] = *reinterpret_cast<const float4*>(conv_w + (size_t)ct * QKV_LEN + ch);
#pragma unroll
        for (int r = 0; r < PREP_TOK + CONV_K - 1; ++r) {
            const int64_t st = tb + r - (CONV_K - 1);
            const float* src;
            if (st >= T) src = nullptr;
            else if (st >= 0) src = qkv + st * QKV_LEN;
            else src = hist + (size_t)((h0 + st + CONV_K) % CONV_K) * QKV_LEN;
            x[r] = src ? *reinterpret_cast<const float4*>(src + ch) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int k = 0; k < PREP_TOK; ++k) {
            const int64_t t = tb + k;
            float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
            if (t < T) {                                // rows of the last chunk past T stay zero
#pragma unroll
                for (int ct = 0; ct < CONV_K; ++ct) {
                    const float4 xv = x[k + ct];
                    acc.x = fmaf(xv.x, w[ct].x, acc.x);
                    acc.y = fmaf(xv.y, w[ct].y, acc.y);
                    acc.z = fmaf(xv.z, w[ct].z, acc.z);
                    acc.w = fmaf(xv.w, w[ct].w, acc.w);
                }
                acc = make_float4(silu_fast(acc.x), silu_fast(acc.y), silu_fast(acc.z), silu_fast(acc.w));
            }
            if (gi < 2 * SSM_HK) {                      // warp-uniform branch: every lane reaches the shuffles
                const float ss = warp_sum(acc.x * acc.x + acc.y * acc.y + acc.z * acc.z + acc.w * acc.w);
                const float inv = 1.0f / sqrtf(ss + 1e-6f);
                acc = make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv);
                if (gi < SSM_HK) acc = make_float4(acc.x * qscale, acc.y * qscale, acc.z * qscale, acc.w * qscale);
            }
            store_split4(dst + (size_t)k * SSM_D, lo_off, lane, acc);
        }
    }
    for (int i = threadIdx.x; i < vc * PREP_TOK; i += blockDim.x) {
        const int vl = i % vc, k = i / vc;
        const int64_t t = tb + k;
        const int vh = vh0 + vl;
        const bool pad = t >= T;     // g = 0, beta = 0 past T
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
    // offset the shared-memory pointer itself (integer arithmetic on the address
    // would turn every later access into a generic one)
    return *reinterpret_cast<S*>(raw + ((1024u - (smem_u32(raw) & 1023u)) & 1023u));
}

// ---------------------------------------------------------------------------
// intra-chunk WY transform: persistent CTAs (8 warps) over the (chunk, local v
// head) items in chunk-major order.  K and Q of the next item are loaded while
// the current one is processed; V goes into the current item's Q rows once
// [K;Q] K^T is done.
// ---------------------------------------------------------------------------
namespace gp {
constexpr int TP = C + 1;        // padded f32 row of the 64x64 matrices (conflict-free column access)
struct alignas(1024) IntraSmem {
    // per buffer: [hi|lo][d-box][row][64]; rows 0-63 = K of the item, 64-127 = Q,
    // then V.  After the W / U0 products a buffer holds the W images (32 KB) then
    // the U0^T image (32 KB) until their bulk store has read them.
    __nv_bfloat16 kq[2][2][2][128][64];
    // A (f32 [64][TP]) and, at U_P, the P image (16 KB), then the block scratch of
    // the inverse; after the inverse: Tm diag(beta e^G) and Tm diag(beta) split
    // images [hi|lo][t][s] (8 KB each) at 0 and 16 KB
    unsigned char u[17408 + 16384];
    float tm[C][TP];                  // (I + A)^-1
    float g[2][C], b[2][C], G[C], eG[C];
    uint64_t bar_kq[2], bar_v, bar_m1, bar_m2;
    uint32_t tmem_base;
};
constexpr uint32_t U_P = 17408;
static_assert(C * TP * 4 <= U_P, "A ends before the P image");
// TMEM columns of the intra kernel
constexpr uint32_t I_KQ = 0, I_W = 64, I_U0 = 128;
}  // namespace gp

__global__ void __launch_bounds__(256, 1) gdn_pf_intra_kernel(const __grid_constant__ CUtensorMap tm_q,
                                                              const __grid_constant__ CUtensorMap tm_k,
                                                              const __grid_constant__ CUtensorMap tm_v, int64_t Tp,
                                                              int item0, int n_items, int vh0, int vc,
                                                              const float* __restrict__ gl,
                                                              const float* __restrict__ bt,
                                                              unsigned char* __restrict__ rec, int* err) {
    using namespace gp;
    using namespace tc;
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    IntraSmem& sm = align1024<IntraSmem>(smem_raw);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    float (*am)[TP] = reinterpret_cast<float (*)[TP]>(sm.u);
    unsigned char* pimg = sm.u + U_P;
    float* xs = reinterpret_cast<float*>(sm.u + U_P);     // block scratch (after the P image is stored)
    unsigned char* tmw = sm.u;                               // [hi|lo][64][64] bf16 (after the inverse)
    unsigned char* tmb = sm.u + 16384;

    if (warp == 0) tmem_alloc(&sm.tmem_base, 256);
    if (tid == 0) {
        mbar_init(&sm.bar_kq[0], 1);
        mbar_init(&sm.bar_kq[1], 1);
        mbar_init(&sm.bar_v, 1);
        mbar_init(&sm.bar_m1, 1);
        mbar_init(&sm.bar_m2, 1);
        fence_mbar_init();
    }
    fence_before_sync();
    __syncthreads();
    fence_after_sync();
    const uint32_t tmem = sm.tmem_base;
    bool ok = true;

    // K, Q, g, beta of item i into buffer b
    auto load_kq = [&](int i, int b) {
        const int c = i / vc, vl = i % vc, kh = (vh0 + vl) % SSM_HK, t0 = c * C;
        mbar_arrive_expect_tx(&sm.bar_kq[b], 8 * 8192 + 2 * 256);
        for (int hl = 0; hl < 2; ++hl)
            for (int db = 0; db < 2; ++db) {
                tma_load_4d(&sm.kq[b][hl][db][0][0], &tm_k, 64 * db, t0, hl, kh, &sm.bar_kq[b]);
                tma_load_4d(&sm.kq[b][hl][db][64][0], &tm_q, 64 * db, t0, hl, kh, &sm.bar_kq[b]);
            }
        bulk_g2s(sm.g[b], gl + (size_t)vl * Tp + t0, 256, &sm.bar_kq[b]);
        bulk_g2s(sm.b[b], bt + (size_t)vl * Tp + t0, 256, &sm.bar_kq[b]);
    };
    if (tid == 0 && item0 + (int)blockIdx.x < n_items) load_kq(item0 + blockIdx.x, 0);

    const int q4 = warp & 3, h = warp >> 2;
    const int row = 32 * q4 + lane;
    const uint32_t lane_addr = tmem + ((uint32_t)(32 * q4) << 16);
    int n = 0;
    for (int i = item0 + blockIdx.x; i < n_items && ok; i += gridDim.x, ++n) {
        const int buf = n & 1;
        const int c = i / vc, vl = i % vc, kh = (vh0 + vl) % SSM_HK;
        unsigned char* R = rec + ((size_t)c * vc + vl) * REC_BYTES;
        const uint32_t ph = (uint32_t)(n & 1);
        wait_or_flag(&sm.bar_kq[buf], (uint32_t)((n >> 1) & 1), err, ok);
        if (!__syncthreads_and(ok)) break;     // every thread takes the same path
        const uint32_t kq_hi = smem_u32(&sm.kq[buf][0][0][0][0]), kq_lo = smem_u32(&sm.kq[buf][1][0][0][0]);
        // ---- [K; Q] K^T  (M 128, N 64, K 128; three split products)
        if (tid == 0) {
            fence_after_sync();
            constexpr uint32_t ID = idesc_bf16(128, 64, false);
            const uint64_t dh = sw128_desc(kq_hi, 16, 1024), dl = sw128_desc(kq_lo, 16, 1024);
#pragma unroll
            for (int pass = 0; pass < 3; ++pass) {
                const uint64_t a = pass == 2 ? dl : dh, bb = pass == 1 ? dl : dh;
#pragma unroll
                for (int ks = 0; ks < 8; ++ks) {
                    const uint64_t off = (uint64_t)(((ks >> 2) * 16384 + (ks & 3) * 32) >> 4);
                    umma_ss(tmem + I_KQ, a + off, bb + off, ID, (pass | ks) != 0);
                }
            }
            umma_commit(&sm.bar_m1);
            // the next item's K/Q go into the other buffer once item n-1's record
            // store (its W/U0 images live there) has read it; P and G of item n-1
            // were waited for after its level-1 inverse
            bulk_wait_read_all();
            if (i + (int)gridDim.x < n_items) load_kq(i + gridDim.x, buf ^ 1);
        }
        if (warp == 1) {   // inclusive cumsum of the 64 log decays (2 per lane)
            const float a0 = sm.g[buf][2 * lane], a1 = sm.g[buf][2 * lane + 1];
            float sum = a0 + a1;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const float y = __shfl_up_sync(0xffffffffu, sum, o);
                if (lane >= o) sum += y;
            }
            const float excl = sum - (a0 + a1);
            sm.G[2 * lane] = excl + a0;
            sm.G[2 * lane + 1] = excl + a0 + a1;
            sm.eG[2 * lane] = expf(excl + a0);
            sm.eG[2 * lane + 1] = expf(excl + a0 + a1);
        }
        wait_or_flag(&sm.bar_m1, ph, err, ok);
        if (!__syncthreads_and(ok)) break;
        fence_after_sync();
        if (tid == 0) {   // V into the Q rows (Q is no longer read)
            mbar_arrive_expect_tx(&sm.bar_v, 4 * 8192);
            for (int hl = 0; hl < 2; ++hl)
                for (int db = 0; db < 2; ++db)
                    tma_load_4d(&sm.kq[buf][hl][db][64][0], &tm_v, 64 * db, c * C, hl, vl, &sm.bar_v);
        }
        // ---- epilogue 1: rows 0-63 -> A (f32, for the inverse), rows 64-127 -> P image
        const float* bcur = sm.b[buf];
        {
            float x[32];
            tmem_ld32(lane_addr + I_KQ + 32 * h, x);
            if (row < C) {
                const int t = row;
                const float bt_ = bcur[t], Gt = sm.G[t];
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    const int s = 32 * h + j;
                    am[t][s] = s < t ? bt_ * __expf(Gt - sm.G[s]) * x[j] : 0.0f;
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
                        const float p0 = s <= t ? __expf(Gt - sm.G[s]) * x[j] : 0.0f;
                        const float p1 = s + 1 <= t ? __expf(Gt - sm.G[s + 1]) * x[j + 1] : 0.0f;
                        split2_bf16(p0, p1, hp[e], lp[e]);
                    }
                    const uint32_t off = sw128_off_b16((uint32_t)t, (uint32_t)(32 * h + 8 * j8));
                    *reinterpret_cast<uint4*>(pimg + off) = hi;
                    *reinterpret_cast<uint4*>(pimg + 8192 + off) = lo;
                }
            }
        }
        fence_proxy_async_smem();
        __syncthreads();
        if (tid == 0) {
            bulk_s2g(R + REC_P, pimg, 16384);
            bulk_s2g(R + REC_G, sm.G, 256);
            bulk_commit();
        }
        // ---- Tm = (I + A)^-1.  Level 1: the four 16x16 diagonal blocks, lane j = column j
        if (warp < 4) {
            if (lane < 16) {
                const int b0 = 16 * warp, j = lane;
                float x[16];
#pragma unroll
                for (int r = 0; r < 16; ++r) {
                    float acc = r == j ? 1.0f : 0.0f;
#pragma unroll
                    for (int q = 0; q < r; ++q) acc = fmaf(-am[b0 + r][b0 + q], x[q], acc);
                    x[r] = acc;
                }
#pragma unroll
                for (int r = 0; r < 16; ++r) sm.tm[b0 + r][b0 + j] = x[r];
            }
        } else {
            // zero the strictly upper blocks (block row I < block column J)
            for (int e = tid - 128; e < 6 * 256; e += 128) {
                const int blk = e >> 8, w = e & 255;
                const int I = blk < 3 ? 0 : (blk < 5 ? 1 : 2);
                const int J = blk < 3 ? blk + 1 : (blk < 5 ? blk - 1 : 3);
                sm.tm[16 * I + (w >> 4)][16 * J + (w & 15)] = 0.0f;
            }
        }
        if (tid == 0) bulk_wait_read_all();   // the P image is read: its bytes become scratch
        __syncthreads();
        // Level 2: T_10 = -T_11 (A_10 T_00) and T_32 = -T_33 (A_32 T_22); two outputs a thread
        {
            const int pr = tid >> 7, idx = tid & 127;
            const int I = 1 + 2 * pr, J = 2 * pr;
            const int r = idx >> 3, c0 = (idx & 7) * 2;
            float* X = xs + pr * 16 * 17;
            float a0 = 0.0f, a1 = 0.0f;
#pragma unroll
            for (int q = 0; q < 16; ++q) {
                const float av = am[16 * I + r][16 * J + q];
                a0 = fmaf(av, sm.tm[16 * J + q][16 * J + c0], a0);
                a1 = fmaf(av, sm.tm[16 * J + q][16 * J + c0 + 1], a1);
            }
            X[r * 17 + c0] = a0;
            X[r * 17 + c0 + 1] = a1;
            __syncthreads();
            float t0v = 0.0f, t1v = 0.0f;
#pragma unroll
            for (int q = 0; q < 16; ++q) {
                const float tv = sm.tm[16 * I + r][16 * I + q];
                t0v = fmaf(tv, X[q * 17 + c0], t0v);
                t1v = fmaf(tv, X[q * 17 + c0 + 1], t1v);
            }
            sm.tm[16 * I + r][16 * J + c0] = -t0v;
            sm.tm[16 * I + r][16 * J + c0 + 1] = -t1v;
        }
        __syncthreads();
        // Level 3: T_21 (rows 32-63, cols 0-31) = -T_2 (A_21 T_1); four outputs a thread
        {
            const int r = tid >> 3, c0 = (tid & 7) * 4;
            float* X = xs;                     // [32][33]
            float a[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll 8
            for (int q = 0; q < 32; ++q) {
                const float av = am[32 + r][q];
#pragma unroll
                for (int e = 0; e < 4; ++e) a[e] = fmaf(av, sm.tm[q][c0 + e], a[e]);
            }
            __syncthreads();                   // every level-2 read of xs is done
#pragma unroll
            for (int e = 0; e < 4; ++e) X[r * 33 + c0 + e] = a[e];
            __syncthreads();
#pragma unroll
            for (int e = 0; e < 4; ++e) a[e] = 0.0f;
#pragma unroll 8
            for (int q = 0; q < 32; ++q) {
                const float tv = sm.tm[32 + r][32 + q];
#pragma unroll
                for (int e = 0; e < 4; ++e) a[e] = fmaf(tv, X[q * 33 + c0 + e], a[e]);
            }
            __syncthreads();                   // A and the scratch are no longer read
#pragma unroll
            for (int e = 0; e < 4; ++e) sm.tm[32 + r][c0 + e] = -a[e];
        }
        __syncthreads();
        // ---- Tm diag(beta e^G) and Tm diag(beta) as split K-major images [t][s]
        for (int e = tid; e < C * 8; e += 256) {
            const int t = e >> 3, j8 = e & 7;
            uint4 wh, wl, bh, bl;
            uint32_t *whp = &wh.x, *wlp = &wl.x, *bhp = &bh.x, *blp = &bl.x;
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const int s2 = 8 * j8 + 2 * k;
                const float v0 = sm.tm[t][s2], v1 = sm.tm[t][s2 + 1];
                const float cb0 = bcur[s2], cb1 = bcur[s2 + 1];
                split2_bf16(v0 * cb0 * sm.eG[s2], v1 * cb1 * sm.eG[s2 + 1], whp[k], wlp[k]);
                split2_bf16(v0 * cb0, v1 * cb1, bhp[k], blp[k]);
            }
            const uint32_t off = sw128_off_b16((uint32_t)t, (uint32_t)(8 * j8));
            *reinterpret_cast<uint4*>(tmw + off) = wh;
            *reinterpret_cast<uint4*>(tmw + 8192 + off) = wl;
            *reinterpret_cast<uint4*>(tmb + off) = bh;
            *reinterpret_cast<uint4*>(tmb + 8192 + off) = bl;
        }
        fence_proxy_async_smem();
        __syncthreads();
        // ---- W^T = K^T TmW^T and U0^T = V^T TmB^T  (M 128 over k / v, N 64, K 64; A MN-major)
        if (tid == 0) {
            if (wait_or_flag(&sm.bar_v, ph, err, ok)) {
                fence_after_sync();
                constexpr uint32_t ID = idesc_bf16(128, 64, false, true);
                // A: rows s (128 B of d each) of the 16 KB d-boxes; K at row 0, V at row 64
                const uint64_t kh_ = sw128_desc(kq_hi, 16384, 1024), kl_ = sw128_desc(kq_lo, 16384, 1024);
                const uint64_t wh_ = sw128_desc(smem_u32(tmw), 16, 1024), wl_ = wh_ + (8192 >> 4);
                const uint64_t bh_ = sw128_desc(smem_u32(tmb), 16, 1024), bl_ = bh_ + (8192 >> 4);
#pragma unroll
                for (int pass = 0; pass < 3; ++pass) {
                    const uint64_t a = pass == 2 ? kl_ : kh_, bb = pass == 1 ? wl_ : wh_;
#pragma unroll
                    for (int ks = 0; ks < 4; ++ks)
                        umma_ss(tmem + I_W, a + (uint64_t)((ks * 2048) >> 4), bb + (uint64_t)((ks * 32) >> 4), ID,
                                (pass | ks) != 0);
                }
#pragma unroll
                for (int pass = 0; pass < 3; ++pass) {
                    const uint64_t a = (pass == 2 ? kl_ : kh_) + (8192 >> 4), bb = pass == 1 ? bl_ : bh_;
#pragma unroll
                    for (int ks = 0; ks < 4; ++ks)
                        umma_ss(tmem + I_U0, a + (uint64_t)((ks * 2048) >> 4), bb + (uint64_t)((ks * 32) >> 4), ID,
                                (pass | ks) != 0);
                }
                umma_commit(&sm.bar_m2);
            }
        }
        wait_or_flag(&sm.bar_m2, ph, err, ok);
        if (!__syncthreads_and(ok)) break;
        fence_after_sync();
        // ---- epilogue 2: W images and the U0^T image into this buffer, then one bulk store
        unsigned char* img = reinterpret_cast<unsigned char*>(&sm.kq[buf][0][0][0][0]);
        {
            float x[32];
            // W^T: lane = k, columns t in [32h, 32h + 32) -> W[t][k]; lane pairs (k, k+1) make one word
            tmem_ld32(lane_addr + I_W + 32 * h, x);
            const uint32_t kb = (uint32_t)row >> 6, kc = (uint32_t)row & 62u;
            const bool odd = (lane & 1) != 0;
#pragma unroll
            for (int j = 0; j < 32; ++j) {
                uint32_t hi, lo;
                split2_bf16(x[j], 0.0f, hi, lo);                   // low halves = this lane's value
                const uint32_t ph_ = __shfl_xor_sync(0xffffffffu, odd ? hi : lo, 1);
                // even lane: (own hi, partner hi) ; odd lane: (partner lo, own lo)
                const uint32_t word = odd ? ((lo & 0xFFFFu) << 16) | (ph_ & 0xFFFFu)
                                          : (hi & 0xFFFFu) | ((ph_ & 0xFFFFu) << 16);
                const uint32_t off = kb * 8192u + sw128_off_b16((uint32_t)(32 * h + j), kc);
                *reinterpret_cast<uint32_t*>(img + (odd ? 16384u : 0u) + off) = word;
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
        if (tid == 0) {
            bulk_s2g(R + REC_W, img, 65536);
            bulk_commit();
        }
        (void)kh;
    }
    if (tid == 0) bulk_wait_all();
    fence_before_sync();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tmem, 256);
}

// ---------------------------------------------------------------------------
// chunk recurrence: one persistent CTA per local v head
// ---------------------------------------------------------------------------
namespace gp {
struct alignas(1024) ChainSmem {
    // B operand of the S product, per chunk parity: [hi|lo][k-box][128 rows][64 k],
    // rows 0-63 = Q of the chunk (TMA), rows 64-127 = W (record).  Once the S product
    // of the chunk is done the buffer stages the chunk's z rows (TMA load, first 32 KB)
    // and its y rows (TMA store, last 32 KB), f32 [64 t][128 v] each.
    unsigned char wq[2][65536];
    // B operand of the state update, per chunk parity: K [hi|lo][d-box][64 t][64 d]
    // (TMA), scaled in place by e^{G_last - G_t}
    unsigned char kd[2][32768];
    unsigned char p[16384];      // record: P images [hi|lo][64 t][64 s]
    float gring[8][C];           // G of chunks c % 8
    float eg[C];                 // e^{G_t} of the chunk in the y epilogue
    float red[4][C];             // per-warp partial sums of y^2 per token
    uint64_t full_wq[2], full_k[2], full_p, full_g[8], full_z[2], wq_free[2];
    uint64_t mma1_done[2], mma3_done[2], mma2_done;
    uint64_t s_ready, u_ready, kd_ready[2], yp_free, yu_free;
    uint32_t tmem_base;
};
// TMEM columns of the chain kernel (512 allocated)
constexpr uint32_t S_ACC = 0;    // f32 state [v lane][k], holds e^{G_last} S between the S epilogue and MMA3
constexpr uint32_t S_HI = 128;   // bf16 pairs of S (A operand), 64 columns
constexpr uint32_t S_LO = 192;
constexpr uint32_t D_YP = 256;   // S Q^T  [v][t]   } one N = 128 product
constexpr uint32_t D_U = 320;    // S W^T  [v][t]   }
constexpr uint32_t U_HI = 384;   // bf16 pairs of U^T (A operand), 32 columns
constexpr uint32_t U_LO = 416;
constexpr uint32_t D_YU = 448;   // U^T P^T [v][t]
// warp roles
constexpr int EY_W0 = 0;         // warps 0-7: y epilogue (gated RMSNorm, store), tokens split in halves
constexpr int E1_W0 = 8;         // warps 8-15: U and S epilogues (the serial path)
constexpr int ES_W0 = 16;        // warps 16-17: K e^{G_last - G} scaling
constexpr int ES_THREADS = 64;
constexpr int LD_W = 18;         // warp 18, lane 0: loads
constexpr int MMA_W = 19;        // warp 19, lane 0: issues the tensor-core products
constexpr int CHAIN_THREADS = 20 * 32;   // 5 warps per SM sub-partition: up to 96 registers a thread
constexpr int BAR_EY = 1;        // named barrier of the y-epilogue warps (0 is __syncthreads)
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


// U0^T of one record, row v, t in [32h, 32h + 32): eight 16-byte chunks whose
// positions in the image are XOR-swizzled by v % 8
__device__ __forceinline__ void load_u0(const unsigned char* rec_u0, int v, int h, float4 (&u)[8]) {
    const unsigned char* row = rec_u0 + (size_t)h * 16384 + (size_t)v * 128;
#pragma unroll
    for (int j = 0; j < 8; ++j) u[j] = __ldg(reinterpret_cast<const float4*>(row + ((j ^ (v & 7)) << 4)));
}

__global__ void __launch_bounds__(gp::CHAIN_THREADS, 1) gdn_pf_chain_kernel(
    const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
    const __grid_constant__ CUtensorMap tm_z, const __grid_constant__ CUtensorMap tm_y, int c0, int NC, int vh0,
    int vc, const unsigned char* __restrict__ rec, float* __restrict__ state, const float* __restrict__ norm_w, int* err) {
    using namespace gp;
    using namespace tc;
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    ChainSmem& sm = align1024<ChainSmem>(smem_raw);
    const int vl = blockIdx.x, tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31;
    const int kh = (vh0 + vl) % SSM_HK;
    // chunks c0 .. c0 + NC - 1 of the sequence; loop counters below are local (0 .. NC - 1)
    auto R = [&](int c) { return rec + ((size_t)(c0 + c) * vc + vl) * REC_BYTES; };

    if (warp == MMA_W) tmem_alloc(&sm.tmem_base, 512);
    if (tid == 0) {
        for (int i = 0; i < 2; ++i) {
            mbar_init(&sm.full_wq[i], 1);
            mbar_init(&sm.full_k[i], 1);
            mbar_init(&sm.mma1_done[i], 1);
            mbar_init(&sm.mma3_done[i], 1);
            mbar_init(&sm.kd_ready[i], ES_THREADS);
        }
        for (int i = 0; i < 8; ++i) mbar_init(&sm.full_g[i], 1);
        mbar_init(&sm.full_p, 1);
        mbar_init(&sm.mma2_done, 1);
        mbar_init(&sm.s_ready, 256);
        mbar_init(&sm.u_ready, 256);
        mbar_init(&sm.yp_free, 256);
        mbar_init(&sm.full_z[0], 1);
        mbar_init(&sm.full_z[1], 1);
        mbar_init(&sm.wq_free[0], 1);
        mbar_init(&sm.wq_free[1], 1);
        mbar_init(&sm.yu_free, 256);
        fence_mbar_init();
    }
    fence_before_sync();
    __syncthreads();
    fence_after_sync();
    const uint32_t tmem = sm.tmem_base;
    bool ok = true;

    if (warp == LD_W) {
        if (lane == 0) {
            // ---------------- loader ----------------
            // Buffers of parity b are reused by chunk c + 2 once chunk c's readers are
            // done: WQ after MMA1(c), KD after MMA3(c) (per-parity barriers, one
            // completion every two chunks); P after MMA2(c-1).  G slots are 8 chunks
            // apart; slot (c+5)%8 held chunk c-3, whose last reader (the y epilogue)
            // finished before MMA1(c-2).
            for (int c = 0; c < NC && c < 5; ++c) {
                mbar_arrive_expect_tx(&sm.full_g[c], 256);
                bulk_g2s(sm.gring[c], R(c) + REC_G, 256, &sm.full_g[c]);
            }
            for (int c = 0; c < NC && ok; ++c) {
                const int b = c & 1;
                const uint32_t pp2 = (uint32_t)(((c - 2) >> 1) & 1);
                const int t0 = (c0 + c) * C;
                // K(c) -> KD[b]
                if (c > 1 && !wait_or_flag(&sm.mma3_done[b], pp2, err, ok)) break;
                mbar_arrive_expect_tx(&sm.full_k[b], 32768);
                for (int hl = 0; hl < 2; ++hl)
                    for (int db = 0; db < 2; ++db)
                        tma_load_4d(sm.kd[b] + hl * 16384 + db * 8192, &tm_k, 64 * db, t0, hl, kh, &sm.full_k[b]);
                // z(c-1) -> WQ[(c-1)%2] once the S product of chunk c-1 is done
                if (c > 0) {
                    const int bp = (c - 1) & 1;
                    if (!wait_or_flag(&sm.mma1_done[bp], (uint32_t)(((c - 1) >> 1) & 1), err, ok)) break;
                    mbar_arrive_expect_tx(&sm.full_z[bp], C * D * 4);
                    tma_load_2d(sm.wq[bp], &tm_z, (vh0 + vl) * D, (c0 + c - 1) * C, &sm.full_z[bp]);
                }
                // G(c+5) into the slot of chunk c-3, whose last reader (the y epilogue) was done
                // before MMA1(c-2)
                if (c + 5 < NC) {
                    const int s = (c + 5) & 7;
                    mbar_arrive_expect_tx(&sm.full_g[s], 256);
                    bulk_g2s(sm.gring[s], R(c + 5) + REC_G, 256, &sm.full_g[s]);
                }
                // Q(c) and W(c) -> WQ[b] once the y rows of chunk c-2 have left it
                if (c > 1 && !wait_or_flag(&sm.wq_free[b], pp2, err, ok)) break;
                mbar_arrive_expect_tx(&sm.full_wq[b], 65536);
                for (int hl = 0; hl < 2; ++hl)
                    for (int kb = 0; kb < 2; ++kb) {
                        unsigned char* box = sm.wq[b] + hl * 32768 + kb * 16384;
                        tma_load_4d(box, &tm_q, 64 * kb, t0, hl, kh, &sm.full_wq[b]);
                        bulk_g2s(box + 8192, R(c) + REC_W + hl * 16384 + kb * 8192, 8192, &sm.full_wq[b]);
                    }
                // P(c)
                if (c > 0 && !wait_or_flag(&sm.mma2_done, (uint32_t)((c - 1) & 1), err, ok)) break;
                mbar_arrive_expect_tx(&sm.full_p, 16384);
                bulk_g2s(sm.p, R(c) + REC_P, 16384, &sm.full_p);
            }
            // z of the last chunk
            if (ok && NC > 0) {
                const int bp = (NC - 1) & 1;
                if (wait_or_flag(&sm.mma1_done[bp], (uint32_t)(((NC - 1) >> 1) & 1), err, ok)) {
                    mbar_arrive_expect_tx(&sm.full_z[bp], C * D * 4);
                    tma_load_2d(sm.wq[bp], &tm_z, (vh0 + vl) * D, (c0 + NC - 1) * C, &sm.full_z[bp]);
                }
            }
        }
    } else if (warp == MMA_W) {
        if (lane == 0) {
            // ---------------- MMA issuer ----------------
            constexpr uint32_t ID128 = idesc_bf16(128, 128, false);
            constexpr uint32_t ID128MN = idesc_bf16(128, 128, true);
            constexpr uint32_t ID64 = idesc_bf16(128, 64, false);
            // descriptors of the buffers' first bytes; an offset of o bytes adds o >> 4
            // (shared-memory addresses stay below 256 KB, inside the 14-bit field)
            const uint64_t dwq0 = sw128_desc(smem_u32(sm.wq[0]), 16, 1024);
            const uint64_t dkd0 = sw128_desc(smem_u32(sm.kd[0]), 8192, 1024);
            const uint64_t dp0 = sw128_desc(smem_u32(sm.p), 16, 1024);
            for (int c = 0; c < NC && ok; ++c) {
                const int b = c & 1;
                const uint32_t ph = (uint32_t)(c & 1), pb = (uint32_t)((c >> 1) & 1);
                // [D_YP | D_U] = S [Q; W]^T  (A = S hi/lo in TMEM, N 128, K 128)
                if (!wait_or_flag(&sm.s_ready, ph, err, ok) || !wait_or_flag(&sm.full_wq[b], pb, err, ok)) break;
                if (c > 0 && !wait_or_flag(&sm.yp_free, (uint32_t)((c - 1) & 1), err, ok)) break;
                fence_after_sync();
#pragma unroll
                for (int pass = 0; pass < 3; ++pass) {
                    const uint32_t a = pass == 2 ? S_LO : S_HI;
                    const uint64_t bd = dwq0 + (uint64_t)((b * 65536 + (pass == 1 ? 32768 : 0)) >> 4);
#pragma unroll
                    for (int ks = 0; ks < 8; ++ks)
                        umma_ts(tmem + D_YP, tmem + a + 8u * ks, bd + (uint64_t)(((ks >> 2) * 16384 + (ks & 3) * 32) >> 4),
                                ID128, (pass | ks) != 0);
                }
                umma_commit(&sm.mma1_done[b]);
                // S_ACC (= e^{G_last} S) += U^T Kd  (A = U hi/lo, B = Kd MN-major, N 128, K 64)
                if (!wait_or_flag(&sm.u_ready, ph, err, ok) || !wait_or_flag(&sm.kd_ready[b], pb, err, ok)) break;
                fence_after_sync();
#pragma unroll
                for (int pass = 0; pass < 3; ++pass) {
                    const uint32_t a = pass == 2 ? U_LO : U_HI;
                    const uint64_t bd = dkd0 + (uint64_t)((b * 32768 + (pass == 1 ? 16384 : 0)) >> 4);
#pragma unroll
                    for (int ks = 0; ks < 4; ++ks)
                        umma_ts(tmem + S_ACC, tmem + a + 8u * ks, bd + (uint64_t)((ks * 2048) >> 4), ID128MN, 1);
                }
                umma_commit(&sm.mma3_done[b]);
                // D_YU = U^T P^T  (B = P images, N 64, K 64)
                if (!wait_or_flag(&sm.full_p, ph, err, ok)) break;
                if (c > 0 && !wait_or_flag(&sm.yu_free, (uint32_t)((c - 1) & 1), err, ok)) break;
                fence_after_sync();
#pragma unroll
                for (int pass = 0; pass < 3; ++pass) {
                    const uint32_t a = pass == 2 ? U_LO : U_HI;
                    const uint64_t bd = dp0 + (uint64_t)((pass == 1 ? 8192 : 0) >> 4);
#pragma unroll
                    for (int ks = 0; ks < 4; ++ks)
                        umma_ts(tmem + D_YU, tmem + a + 8u * ks, bd + (uint64_t)((ks * 32) >> 4), ID64, (pass | ks) != 0);
                }
                umma_commit(&sm.mma2_done);
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
#pragma unroll 1
            for (int piece = 0; piece < 4; ++piece) {
                const int k0 = 64 * h + 16 * piece;
                uint32_t hi[8], lo[8], sc[16];
#pragma unroll
                for (int j4 = 0; j4 < 4; ++j4) {
                    const float4 s4 = *reinterpret_cast<const float4*>(Sg + k0 + 4 * j4);
                    split2_bf16(s4.x, s4.y, hi[2 * j4], lo[2 * j4]);
                    split2_bf16(s4.z, s4.w, hi[2 * j4 + 1], lo[2 * j4 + 1]);
                    sc[4 * j4] = __float_as_uint(s4.x * e0);
                    sc[4 * j4 + 1] = __float_as_uint(s4.y * e0);
                    sc[4 * j4 + 2] = __float_as_uint(s4.z * e0);
                    sc[4 * j4 + 3] = __float_as_uint(s4.w * e0);
                }
                tmem_st8_async(la + S_HI + (uint32_t)(k0 >> 1), hi);
                tmem_st8_async(la + S_LO + (uint32_t)(k0 >> 1), lo);
                tmem_st16_async(la + S_ACC + (uint32_t)k0, sc);
                tmem_wait_st();
            }
        }
        fence_before_sync();
        mbar_arrive(&sm.s_ready);
        float4 u0[8];
        load_u0(R(0) + REC_U0, v, h, u0);
        for (int c = 0; c < NC && ok; ++c) {
            const int b = c & 1;
            const uint32_t pb = (uint32_t)((c >> 1) & 1);
            // U^T = U0^T - S W^T  -> bf16 pairs (columns t in [32h, 32h + 32))
            if (!wait_or_flag(&sm.mma1_done[b], pb, err, ok)) break;
            fence_after_sync();
            {
                uint32_t r[32];
                tmem_ld32_async(la + D_U + 32u * h, r);
                tmem_wait_ld();
                uint32_t hi[16], lo[16];
#pragma unroll
                for (int j4 = 0; j4 < 8; ++j4) {
                    split2_bf16(u0[j4].x - __uint_as_float(r[4 * j4]), u0[j4].y - __uint_as_float(r[4 * j4 + 1]),
                                hi[2 * j4], lo[2 * j4]);
                    split2_bf16(u0[j4].z - __uint_as_float(r[4 * j4 + 2]), u0[j4].w - __uint_as_float(r[4 * j4 + 3]),
                                hi[2 * j4 + 1], lo[2 * j4 + 1]);
                }
                tmem_st16_async(la + U_HI + 16u * h, hi);
                tmem_st16_async(la + U_LO + 16u * h, lo);
                tmem_wait_st();
            }
            fence_before_sync();
            mbar_arrive(&sm.u_ready);
            // the next chunk's U0^T row: into L2 now, into registers after the S epilogue
            if (c + 1 < NC)
                asm volatile("prefetch.global.L2 [%0];" ::"l"(R(c + 1) + REC_U0 + (size_t)h * 16384 + (size_t)v * 128));
            // S epilogue: S_{c+1} -> S_HI/S_LO and S_ACC <- e^{G_last(c+1)} S_{c+1}; or the final state
            if (!wait_or_flag(&sm.mma3_done[b], pb, err, ok)) break;
            fence_after_sync();
            const bool last = c + 1 == NC;
            float e1 = 1.0f;
            if (!last) {
                const int s = (c + 1) & 7;
                if (!wait_or_flag(&sm.full_g[s], (uint32_t)(((c + 1) >> 3) & 1), err, ok)) break;
                e1 = expf(sm.gring[s][C - 1]);
            }
#pragma unroll 1
            for (int piece = 0; piece < 4; ++piece) {
                const int k0 = 64 * h + 16 * piece;
                uint32_t r[16];
                tmem_ld16_async(la + S_ACC + (uint32_t)k0, r);
                tmem_wait_ld();
                if (last) {
#pragma unroll
                    for (int j4 = 0; j4 < 4; ++j4)
                        *reinterpret_cast<float4*>(Sg + k0 + 4 * j4) =
                            make_float4(__uint_as_float(r[4 * j4]), __uint_as_float(r[4 * j4 + 1]),
                                        __uint_as_float(r[4 * j4 + 2]), __uint_as_float(r[4 * j4 + 3]));
                } else {
                    uint32_t hi[8], lo[8];
#pragma unroll
                    for (int j = 0; j < 8; ++j)
                        split2_bf16(__uint_as_float(r[2 * j]), __uint_as_float(r[2 * j + 1]), hi[j], lo[j]);
                    tmem_st8_async(la + S_HI + (uint32_t)(k0 >> 1), hi);
                    tmem_st8_async(la + S_LO + (uint32_t)(k0 >> 1), lo);
#pragma unroll
                    for (int j = 0; j < 16; ++j) r[j] = __float_as_uint(__uint_as_float(r[j]) * e1);
                    tmem_st16_async(la + S_ACC + (uint32_t)k0, r);
                }
            }
            if (!last) {
                tmem_wait_st();
                fence_before_sync();
                mbar_arrive(&sm.s_ready);
                load_u0(R(c + 1) + REC_U0, v, h, u0);
            }
        }
    } else if (warp >= ES_W0 && warp < LD_W) {
        // ---------------- K e^{G_last - G}, in place ----------------
        const int et = tid - ES_W0 * 32;
        for (int c = 0; c < NC && ok; ++c) {
            const int b = c & 1, s = c & 7;
            if (!wait_or_flag(&sm.full_g[s], (uint32_t)((c >> 3) & 1), err, ok)) break;
            if (!wait_or_flag(&sm.full_k[b], (uint32_t)((c >> 1) & 1), err, ok)) break;
            const float* G = sm.gring[s];
            const float Gl = G[C - 1];
            unsigned char* img = sm.kd[b];
            for (int i = et; i < 1024; i += ES_THREADS) {   // 16-byte chunks of the hi image
                const uint32_t off = (uint32_t)i * 16u;
                const float sc = __expf(Gl - G[(off & 8191u) >> 7]);
                uint4 hq = *reinterpret_cast<const uint4*>(img + off);
                uint4 lq = *reinterpret_cast<const uint4*>(img + 16384 + off);
                uint32_t* hp = &hq.x;
                uint32_t* lp = &lq.x;
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float a = (bf16_lo_f(hp[e]) + bf16_lo_f(lp[e])) * sc;
                    const float bb = (bf16_hi_f(hp[e]) + bf16_hi_f(lp[e])) * sc;
                    split2_bf16(a, bb, hp[e], lp[e]);
                }
                *reinterpret_cast<uint4*>(img + off) = hq;
                *reinterpret_cast<uint4*>(img + 16384 + off) = lq;
            }
            fence_proxy_async_smem();
            mbar_arrive(&sm.kd_ready[b]);
        }
    } else {
        // ---------------- y epilogue: y = e^G o (S Q^T) + U^T P^T, gated RMSNorm, store ----------------
        const int q4 = (warp - EY_W0) & 3, th = (warp - EY_W0) >> 2;   // lanes 32 q4.., tokens [32 th, 32 th + 32)
        const int v = 32 * q4 + lane;
        const uint32_t la = tmem + ((uint32_t)(32 * q4) << 16);
        const float wv = norm_w[v];
        for (int c = 0; c < NC; ++c) {
            const int b = c & 1, s = c & 7;
            // S Q^T of the chunk, as soon as the S product is done
            bool got = ok && wait_or_flag(&sm.full_g[s], (uint32_t)((c >> 3) & 1), err, ok) &&
                       wait_or_flag(&sm.mma1_done[b], (uint32_t)((c >> 1) & 1), err, ok);
            if (!named_bar_and(BAR_EY, 256, got)) {
                ok = false;
                break;
            }
            fence_after_sync();
            float y[32];
            {
                uint32_t r[32];
                tmem_ld32_async(la + D_YP + 32u * th, r);
                tmem_wait_ld();
#pragma unroll
                for (int j = 0; j < 32; ++j) y[j] = __uint_as_float(r[j]);
            }
            if (tid < C) sm.eg[tid] = __expf(sm.gring[s][tid]);
            fence_before_sync();
            mbar_arrive(&sm.yp_free);
            got = ok && wait_or_flag(&sm.mma2_done, (uint32_t)(c & 1), err, ok);
            if (!named_bar_and(BAR_EY, 256, got)) {
                ok = false;
                break;
            }
            fence_after_sync();
            {
                uint32_t r[32];
                tmem_ld32_async(la + D_YU + 32u * th, r);
                tmem_wait_ld();
#pragma unroll
                for (int j = 0; j < 32; ++j) y[j] = fmaf(sm.eg[32 * th + j], y[j], __uint_as_float(r[j]));
            }
            fence_before_sync();
            mbar_arrive(&sm.yu_free);
            // sum over this warp's 32 v of y^2 per token: lane L ends with token 32 th + L
            float a[16];
            {
                const bool up = (lane & 16) != 0;
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    const float lo2 = y[j] * y[j], hi2 = y[j + 16] * y[j + 16];
                    a[j] = (up ? hi2 : lo2) + __shfl_xor_sync(0xffffffffu, up ? lo2 : hi2, 16);
                }
            }
            bfly_reduce<16, 8>(a, lane);
            bfly_reduce<8, 4>(a, lane);
            bfly_reduce<4, 2>(a, lane);
            bfly_reduce<2, 1>(a, lane);
            sm.red[q4][32 * th + lane] = a[0];
            tc::named_bar_sync(BAR_EY, 256);
            const int tt = 32 * th + lane;
            const float inv_l = 1.0f / sqrtf(((sm.red[0][tt] + sm.red[1][tt]) + (sm.red[2][tt] + sm.red[3][tt])) /
                                                 (float)D + 1e-6f);
            // z rows of the chunk in WQ[b] (TMA, zero past T); y rows staged behind them
            got = ok && wait_or_flag(&sm.full_z[b], (uint32_t)((c >> 1) & 1), err, ok);
            if (!named_bar_and(BAR_EY, 256, got)) {
                ok = false;
                break;
            }
            const float* zt = reinterpret_cast<const float*>(sm.wq[b]);
            float* yt = reinterpret_cast<float*>(sm.wq[b] + 32768);
#pragma unroll
            for (int j = 0; j < 32; ++j) {
                const int t = 32 * th + j;
                const float inv = __shfl_sync(0xffffffffu, inv_l, j);
                yt[t * D + v] = ((y[j] * inv) * wv) * silu_fast(zt[t * D + v]);
            }
            fence_proxy_async_smem();
            tc::named_bar_sync(BAR_EY, 256);
            if (tid == 0) {
                // rows past T are clipped by the tensor store
                tma_store_2d(&tm_y, vl * D, (c0 + c) * C, yt);
                bulk_commit();
                bulk_wait_read_all();
                mbar_arrive(&sm.wq_free[b]);
            }
        }
    }
    fence_before_sync();
    __syncthreads();
    if (warp == MMA_W) tmem_dealloc(tmem, 512);
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
// f32 [rows][cols] with (128 x 64) boxes, no swizzle: the z rows of a head and
// chunk (TMA load, zero past the last row) and the y rows (TMA store, clipped)
bool make_rows_map(CUtensorMap* m, const float* base, int64_t rows, int64_t cols) {
    EncodeTiledFn fn = tensor_map_encoder();
    if (!fn) return false;
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)cols * 4};
    cuuint32_t box[2] = {(cuuint32_t)SSM_D, (cuuint32_t)gp::C};
    cuuint32_t estr[2] = {1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}
size_t round_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// Chunk segments of the pipelined prefill, as boundaries b[0] = 0 < ... < b[n] = NC.
// One segment when the sequence is short (under 16 chunks) or the chain kernels
// would leave too few SMs for the intra-chunk kernels.  Otherwise the segments
// grow from the end backwards (NC/16, doubling, at most NC/4): the chain work
// of the last segment is the only part not overlapped with intra-chunk work.
int pf_segments(int NC, int vc, int n_sm, int* b) {
    b[0] = 0;
    if (NC < 16 || 2 * vc > n_sm) {
        b[1] = NC;
        return 1;
    }
    int sizes[PF_MAX_SEGMENTS];
    int n = 0, rem = NC, sz = std::max(2, NC / 16);
    const int cap = std::max(sz, NC / 4);
    while (rem > 0 && n < PF_MAX_SEGMENTS) {
        const int take = std::min(sz, rem);
        sizes[n++] = take;
        rem -= take;
        sz = std::min(2 * sz, cap);
    }
    sizes[n - 1] += rem;   // whatever is left joins the first segment
    for (int k = 0; k < n; ++k) b[k + 1] = b[k] + sizes[n - 1 - k];
    return n;
}
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

    CUtensorMap mq, mk, mv, mz, my;
    if (!make_split_map(&mq, qs, Tp, SSM_HK) || !make_split_map(&mk, ks, Tp, SSM_HK) ||
        !make_split_map(&mv, vs, Tp, vc) || !make_rows_map(&mz, z, T, INNER) || !make_rows_map(&my, y, T, (int64_t)vc * D))
        return cudaErrorInvalidValue;

    gdn_pf_prep_kernel<<<(unsigned)(Tp / PREP_TOK), 256, 0, st>>>(T, Tp, vh0, vc, h0, qkv, slot.hist, L.conv_w, L.ssm_a,
                                                                  L.dt_bias, alpha, beta, qs, ks, vs, gl, bt);
    gdn_pf_ring_kernel<<<(unsigned)(T < CONV_K ? T : CONV_K), 256, 0, st>>>(T, h0, qkv, slot.hist);
    const int smem_i = (int)sizeof(IntraSmem) + 1024;
    e = cudaFuncSetAttribute(gdn_pf_intra_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_i);
    if (e != cudaSuccess) return e;
    const int smem_c = (int)sizeof(ChainSmem) + 1024;
    e = cudaFuncSetAttribute(gdn_pf_chain_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_c);
    if (e != cudaSuccess) return e;
    int bounds[PF_MAX_SEGMENTS + 1];
    const int nseg = pf_segments(NC, vc, ctx->n_sm, bounds);
    if (nseg == 1) {
        const int n_items = NC * vc;
        gdn_pf_intra_kernel<<<std::min(n_items, ctx->n_sm), 256, smem_i, st>>>(mq, mk, mv, Tp, 0, n_items, vh0, vc, gl,
                                                                              bt, rec, ctx->d_err);
        gdn_pf_chain_kernel<<<vc, CHAIN_THREADS, smem_c, st>>>(mq, mk, mz, my, 0, NC, vh0, vc, rec, slot.state,
                                                               L.norm_w, ctx->d_err);
        *n_launch += 4;
        return cudaGetLastError();
    }
    // Pipelined: the intra-chunk kernels of segment k + 1 (side stream, n_sm - vc
    // CTAs) run while the chain kernel of segment k (this stream, vc CTAs) runs on
    // the other SMs.  Only stream order and events connect them; no kernel waits
    // on another.
    cudaStream_t side = ctx->pf_side;
    if ((e = cudaEventRecord(ctx->pf_ev[0], st)) != cudaSuccess) return e;
    if ((e = cudaStreamWaitEvent(side, ctx->pf_ev[0], 0)) != cudaSuccess) return e;
    const int grid_i = ctx->n_sm - vc;
    for (int k = 0; k < nseg; ++k) {
        const int i0 = bounds[k] * vc, i1 = bounds[k + 1] * vc;
        gdn_pf_intra_kernel<<<std::min(i1 - i0, grid_i), 256, smem_i, side>>>(mq, mk, mv, Tp, i0, i1, vh0, vc, gl, bt,
                                                                             rec, ctx->d_err);
        if ((e = cudaEventRecord(ctx->pf_ev[k + 1], side)) != cudaSuccess) return e;
    }
    for (int k = 0; k < nseg; ++k) {
        if ((e = cudaStreamWaitEvent(st, ctx->pf_ev[k + 1], 0)) != cudaSuccess) return e;
        gdn_pf_chain_kernel<<<vc, CHAIN_THREADS, smem_c, st>>>(mq, mk, mz, my, bounds[k], bounds[k + 1] - bounds[k],
                                                               vh0, vc, rec, slot.state, L.norm_w, ctx->d_err);
    }
    *n_launch += 2 + 2 * nseg;
    return cudaGetLastError();
}

}  // namespace dz
