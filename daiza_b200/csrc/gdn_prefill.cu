// gdn_prefill.cu -- chunked (C = 64) Gated DeltaNet prefill.
//
// Reference: Daiza-engine/src/model/forward.rs:897-1059 -- Phase A (conv1d from
// in-batch rows or pre-batch ring slots (h0+t+ct+1)%4, SiLU, L2-norm q/k,
// q *= 1/sqrt(128), silu(z)), the ring update (last min(4,T) rows, head =
// (h0+T)%4), and Phase B: per v head a chain over t of the fused row pass
// (model/ssm.rs:378-418) followed by the gated RMSNorm (ssm.rs:294-334).
//
// The token recurrence  S_t = e^{g_t} S_{t-1} + u_t k_t^T,
//                        u_t = beta_t (v_t - e^{g_t} S_{t-1} k_t),  y_t = S_t q_t
// is evaluated chunk by chunk (WY / UT form).  With G the in-chunk cumulative
// log decay, Gam_ts = e^{G_t - G_s}, A = strict_lower(beta_t Gam_ts k_t.k_s) and
// Tm = (I + A)^-1:
//   U0 = Tm diag(beta) V,   W = Tm diag(beta e^G) K                (intra, parallel)
//   U  = U0 - W S0^T
//   Y  = diag(e^G) Q S0^T + (lower_incl(Gam) o Q K^T) U
//   S_C = e^{G_last} S0 + U^T diag(e^{G_last - G}) K                 (inter, sequential)
// All exponents are <= 0 (no overflow).  Kernels:
//   gdn_pf_conv   per token: conv + SiLU + L2 norms + gates (log decay, beta)
//   gdn_pf_ring   ring-buffer update (after every conv read)
//   gdn_pf_intra  per (chunk, v head): G, K K^T, Q K^T, Tm by forward
//                 substitution, W, U0, Q e^G, K e^{G_last-G}
//   gdn_pf_inter  per (v head, 32-row block of S): the chunk recurrence
//   gdn_pf_gate   per token: y * inv_rms * w * silu(z)
#include <cstddef>

#include "dz_internal.h"

namespace dz {

namespace gp {
constexpr int C = 64;            // chunk length
constexpr int D = SSM_D;         // 128
constexpr int KP = D + 4;        // padded smem row (floats) for 128-wide rows
constexpr int MP = C + 1;        // padded smem row for 64x64 matrices
constexpr int VB = 16;           // state rows per inter CTA
// Row strides that make warp-level tensor-core fragment reads bank-conflict
// free: A / transposed-B fragments want a stride == 4 (mod 32) floats,
// row-major B fragments a stride == 8 (mod 32).
constexpr int SA = D + 4;    // 132
constexpr int SB = D + 8;    // 136
constexpr int SP = C + 4;    // 68
// per (chunk, v head) record, rows already at the padded strides so that the
// inter kernel moves each operand with ONE bulk copy:
//   X [128][SA] (rows 0..63 = W, 64..127 = Q e^G), U0 [D/VB v-blocks][64][VB],
//   Kd [64][SB], P [64][SP], e^{G_last} (+3 pad)
constexpr size_t OFF_X = 0, OFF_U0 = OFF_X + 2 * C * SA, OFF_KD = OFF_U0 + C * D, OFF_P = OFF_KD + C * SB,
                 OFF_EG = OFF_P + C * SP, REC = OFF_EG + 4;
static_assert(REC % 4 == 0 && OFF_U0 % 4 == 0 && OFF_KD % 4 == 0 && OFF_P % 4 == 0, "16-byte aligned fields");
}  // namespace gp

// ---------------------------------------------------------------------------
// Phase A: conv1d + SiLU + L2 norms + gates, one CTA per token
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) gdn_pf_conv_kernel(int64_t T, int vh0, int vc, int h0,
                                                          const float* __restrict__ qkv,
                                                          const float* __restrict__ hist,
                                                          const float* __restrict__ conv_w,
                                                          const float* __restrict__ ssm_a,
                                                          const float* __restrict__ dt_bias,
                                                          const float* __restrict__ alpha,
                                                          const float* __restrict__ beta, float* __restrict__ qn,
                                                          float* __restrict__ kn, float* __restrict__ vv,
                                                          float* __restrict__ gl, float* __restrict__ bt) {
    const int64_t t = blockIdx.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const float qscale = 1.0f / sqrtf((float)SSM_D);
    for (int gi = warp; gi < 2 * SSM_HK + vc; gi += 8) {
        int cb;
        if (gi < SSM_HK) cb = gi * SSM_D;                               // q head
        else if (gi < 2 * SSM_HK) cb = QKD + (gi - SSM_HK) * SSM_D;     // k head
        else cb = 2 * QKD + (vh0 + gi - 2 * SSM_HK) * SSM_D;            // v head
        const int ch = cb + 4 * lane;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
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
            float inv = 1.0f / sqrtf(ss + 1e-6f);
            const bool is_q = gi < SSM_HK;
            const int kh = is_q ? gi : gi - SSM_HK;
            acc = make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv);
            if (is_q) acc = make_float4(acc.x * qscale, acc.y * qscale, acc.z * qscale, acc.w * qscale);
            float* dst = (is_q ? qn : kn) + ((size_t)t * SSM_HK + kh) * SSM_D;
            reinterpret_cast<float4*>(dst)[lane] = acc;
        } else {
            const int vl = gi - 2 * SSM_HK;
            reinterpret_cast<float4*>(vv + ((size_t)t * vc + vl) * SSM_D)[lane] = acc;
        }
    }
    for (int vl = threadIdx.x; vl < vc; vl += blockDim.x) {
        const int vh = vh0 + vl;
        gl[(size_t)t * vc + vl] = ssm_a[vh] * softplus_ref(alpha[(size_t)t * SSM_HV + vh] + dt_bias[vh]);
        bt[(size_t)t * vc + vl] = sigmoidf_acc(beta[(size_t)t * SSM_HV + vh]);
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

// ---------------------------------------------------------------------------
// warp-level tensor-core tiles: mma m16n8k8 TF32 with f32 accumulation and a
// three-product hi/lo split (a*b ~ ah*bh + ah*bl + al*bh) that keeps the
// products at f32-level accuracy.  Fragment maps (g = lane/4, t = lane%4):
//   A[m][k]: a0 (g,t) a1 (g+8,t) a2 (g,t+4) a3 (g+8,t+4)
//   B[k][n]: b0 (t,g) b1 (t+4,g)        C: c0 (g,2t) c1 (g,2t+1) c2 (g+8,2t) c3 (g+8,2t+1)
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mma_tf32(float (&d)[4], const uint32_t (&a)[4], const uint32_t (&b)[2]) {
    asm volatile(
        "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}
// hi = the 19 leading bits (what a TF32 operand keeps), lo = the exact
// remainder; the MMA itself drops the low bits of lo.
struct FA { uint32_t h[4], l[4]; };
struct FB { uint32_t h[2], l[2]; };
__device__ __forceinline__ void split1(float x, uint32_t& h, uint32_t& l) {
    h = __float_as_uint(x) & 0xFFFFE000u;
    l = __float_as_uint(x - __uint_as_float(h));
}
__device__ __forceinline__ FA split_a(float a0, float a1, float a2, float a3) {
    FA f;
    split1(a0, f.h[0], f.l[0]);
    split1(a1, f.h[1], f.l[1]);
    split1(a2, f.h[2], f.l[2]);
    split1(a3, f.h[3], f.l[3]);
    return f;
}
__device__ __forceinline__ FB split_b(float b0, float b1) {
    FB f;
    split1(b0, f.h[0], f.l[0]);
    split1(b1, f.h[1], f.l[1]);
    return f;
}
__device__ __forceinline__ void mma3(float (&d)[4], const FA& a, const FB& b) {
    mma_tf32(d, a.l, b.h);
    mma_tf32(d, a.h, b.l);
    mma_tf32(d, a.h, b.h);
}

// ---------------------------------------------------------------------------
// intra-chunk WY transform, one CTA (8 warps) per (chunk, local v head)
// ---------------------------------------------------------------------------
namespace gp {
constexpr int SM = C + 4;    // 64-wide matrices read as A fragments
}
struct IntraSmem {
    float K[gp::C][gp::SA];
    float Q[gp::C][gp::SA];
    float V[gp::C][gp::SB];
    float Am[gp::C][gp::SM];   // strictly lower beta_t Gam_ts k_t.k_s
    float Tm[gp::C][gp::SM];   // (I + Am)^-1
    float G[gp::C], b[gp::C], eG[gp::C], cw[gp::C], cu[gp::C];
};

__global__ void __launch_bounds__(256) gdn_pf_intra_kernel(int64_t T, int vh0, int vc, const float* __restrict__ qn,
                                                           const float* __restrict__ kn, const float* __restrict__ vv,
                                                           const float* __restrict__ gl, const float* __restrict__ bt,
                                                           float* __restrict__ rec) {
    using namespace gp;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    IntraSmem& sm = *reinterpret_cast<IntraSmem*>(smem_raw);
    const int c = blockIdx.x, vl = blockIdx.y, tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31, g = lane >> 2, t4 = lane & 3;
    const int vh = vh0 + vl, kh = vh % SSM_HK;
    const int64_t t0 = (int64_t)c * C;
    const int n = (int)(T - t0 < C ? T - t0 : C);
    float* out = rec + ((size_t)c * vc + vl) * REC;

    for (int i = tid; i < C * (D / 4); i += 256) {
        const int r = i / (D / 4), c4 = i % (D / 4);
        float4 k4 = make_float4(0.f, 0.f, 0.f, 0.f), q4 = k4, v4 = k4;
        if (r < n) {
            k4 = reinterpret_cast<const float4*>(kn + ((size_t)(t0 + r) * SSM_HK + kh) * D)[c4];
            q4 = reinterpret_cast<const float4*>(qn + ((size_t)(t0 + r) * SSM_HK + kh) * D)[c4];
            v4 = reinterpret_cast<const float4*>(vv + ((size_t)(t0 + r) * vc + vl) * D)[c4];
        }
        *reinterpret_cast<float4*>(&sm.K[r][4 * c4]) = k4;
        *reinterpret_cast<float4*>(&sm.Q[r][4 * c4]) = q4;
        *reinterpret_cast<float4*>(&sm.V[r][4 * c4]) = v4;
    }
    if (warp == 0) {   // inclusive cumsum of the 64 log decays (2 per lane)
        const float a0 = lane * 2 < n ? gl[(size_t)(t0 + 2 * lane) * vc + vl] : 0.0f;
        const float a1 = lane * 2 + 1 < n ? gl[(size_t)(t0 + 2 * lane + 1) * vc + vl] : 0.0f;
        float s = a0 + a1;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const float y = __shfl_up_sync(0xffffffffu, s, o);
            if (lane >= o) s += y;
        }
        const float excl = s - (a0 + a1);
        sm.G[2 * lane] = excl + a0;
        sm.G[2 * lane + 1] = excl + a0 + a1;
        sm.b[2 * lane] = lane * 2 < n ? bt[(size_t)(t0 + 2 * lane) * vc + vl] : 0.0f;
        sm.b[2 * lane + 1] = lane * 2 + 1 < n ? bt[(size_t)(t0 + 2 * lane + 1) * vc + vl] : 0.0f;
    }
    __syncthreads();
    const float G_last = sm.G[n - 1];
    if (tid < C) {
        const float e = expf(sm.G[tid]);
        sm.eG[tid] = e;
        sm.cw[tid] = sm.b[tid] * e;    // W coefficients   beta e^G
        sm.cu[tid] = sm.b[tid];        // U0 coefficients  beta
    }
    __syncthreads();
    // X rows 64..127 = Q e^G ; Kd = K e^{G_last - G}
    for (int i = tid; i < C * (D / 4); i += 256) {
        const int r = i / (D / 4), c4 = i % (D / 4);
        const float eq = sm.eG[r], ek = expf(G_last - sm.G[r]);
        const float4 q4 = *reinterpret_cast<const float4*>(&sm.Q[r][4 * c4]);
        const float4 k4 = *reinterpret_cast<const float4*>(&sm.K[r][4 * c4]);
        *reinterpret_cast<float4*>(out + OFF_X + (size_t)(C + r) * SA + 4 * c4) =
            make_float4(q4.x * eq, q4.y * eq, q4.z * eq, q4.w * eq);
        *reinterpret_cast<float4*>(out + OFF_KD + (size_t)r * SB + 4 * c4) =
            make_float4(k4.x * ek, k4.y * ek, k4.z * ek, k4.w * ek);
    }
    if (tid == 0) out[OFF_EG] = expf(G_last);

    // ---- [K; Q] K^T on tensor tiles: warp w owns stacked rows 16w..16w+15, 8 n-tiles
    {
        const int m0 = (warp & 3) * 16;
        float (*A)[SA] = warp < 4 ? sm.K : sm.Q;
        float acc[8][4];
#pragma unroll
        for (int j = 0; j < 8; ++j)
#pragma unroll
            for (int e = 0; e < 4; ++e) acc[j][e] = 0.0f;
#pragma unroll 2
        for (int k0 = 0; k0 < D; k0 += 8) {
            const FA a = split_a(A[m0 + g][k0 + t4], A[m0 + g + 8][k0 + t4], A[m0 + g][k0 + t4 + 4],
                                 A[m0 + g + 8][k0 + t4 + 4]);
#pragma unroll
            for (int j = 0; j < 8; ++j) mma3(acc[j], a, split_b(sm.K[8 * j + g][k0 + t4], sm.K[8 * j + g][k0 + t4 + 4]));
        }
        // epilogue: rows of K K^T -> Am (strict lower, beta Gam); rows of Q K^T -> P (lower incl.)
#pragma unroll
        for (int j = 0; j < 8; ++j) {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int i = m0 + g + (e >> 1) * 8;
                const int s = 8 * j + 2 * t4 + (e & 1);
                const float gam = s <= i ? expf(sm.G[i] - sm.G[s]) : 0.0f;
                if (warp < 4) sm.Am[i][s] = s < i ? sm.b[i] * gam * acc[j][e] : 0.0f;
                else out[OFF_P + i * SP + s] = gam * acc[j][e];
            }
        }
    }
    __syncthreads();
    // ---- Tm = (I + Am)^-1, blocked 16x16.  Diagonal blocks: warp b, forward substitution.
    if (warp < 4) {
        const int b0 = 16 * warp;
        for (int i = 0; i < 16; ++i) {
            if (lane < 16) {
                const int j = lane;
                float x = (i == j) ? 1.0f : 0.0f;
                for (int s = j; s < i; ++s) x = fmaf(-sm.Am[b0 + i][b0 + s], sm.Tm[b0 + s][b0 + j], x);
                sm.Tm[b0 + i][b0 + j] = (j <= i) ? x : 0.0f;
                // zero the strictly upper blocks of this block row
                for (int jj = b0 + 16; jj < C; jj += 16) sm.Tm[b0 + i][jj + j] = 0.0f;
            }
            __syncwarp();
        }
    }
    __syncthreads();
    // off-diagonal blocks by block diagonal d: T_IJ = -T_II * sum_{K=J}^{I-1} A_IK T_KJ
    for (int d = 1; d < 4; ++d) {
        if (warp < 4 - d) {
            const int J = warp, I = warp + d;
            float m[8];
            // lane computes 8 entries of M (16x16): rows r = lane/2, cols 8*(lane%2)..+8
            const int r = lane >> 1, cb = 8 * (lane & 1);
#pragma unroll
            for (int e = 0; e < 8; ++e) m[e] = 0.0f;
            for (int Kb = J; Kb < I; ++Kb)
                for (int s = 0; s < 16; ++s) {
                    const float a = sm.Am[16 * I + r][16 * Kb + s];
#pragma unroll
                    for (int e = 0; e < 8; ++e) m[e] = fmaf(a, sm.Tm[16 * Kb + s][16 * J + cb + e], m[e]);
                }
            // stash M in the (still zero) target block, then T_IJ = -T_II M
#pragma unroll
            for (int e = 0; e < 8; ++e) sm.Tm[16 * I + r][16 * J + cb + e] = m[e];
            __syncwarp();
            float o[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) o[e] = 0.0f;
            for (int s = 0; s <= r; ++s) {
                const float tii = sm.Tm[16 * I + r][16 * I + s];
#pragma unroll
                for (int e = 0; e < 8; ++e) o[e] = fmaf(tii, sm.Tm[16 * I + s][16 * J + cb + e], o[e]);
            }
            __syncwarp();
#pragma unroll
            for (int e = 0; e < 8; ++e) sm.Tm[16 * I + r][16 * J + cb + e] = -o[e];
        }
        __syncthreads();
    }
    // ---- [W | U0] = Tm [beta e^G K | beta V]  (64 x 256): warp -> m-tile (warp&3), 16 n-tiles of half (warp>>2)
    {
        const int m0 = (warp & 3) * 16;
        const bool is_u = warp >= 4;
        const float* coef = is_u ? sm.cu : sm.cw;
        float acc[16][4];
#pragma unroll
        for (int j = 0; j < 16; ++j)
#pragma unroll
            for (int e = 0; e < 4; ++e) acc[j][e] = 0.0f;
        for (int k0 = 0; k0 < C; k0 += 8) {
            const FA a = split_a(sm.Tm[m0 + g][k0 + t4], sm.Tm[m0 + g + 8][k0 + t4], sm.Tm[m0 + g][k0 + t4 + 4],
                                 sm.Tm[m0 + g + 8][k0 + t4 + 4]);
            const float c0 = coef[k0 + t4], c1 = coef[k0 + t4 + 4];
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                const FB bb = is_u ? split_b(c0 * sm.V[k0 + t4][8 * j + g], c1 * sm.V[k0 + t4 + 4][8 * j + g])
                                   : split_b(c0 * sm.K[k0 + t4][8 * j + g], c1 * sm.K[k0 + t4 + 4][8 * j + g]);
                mma3(acc[j], a, bb);
            }
        }
#pragma unroll
        for (int j = 0; j < 16; ++j) {
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int i = m0 + g + 8 * h;
                const int col = 8 * j + 2 * t4;
                const float2 v2 = make_float2(acc[j][2 * h], acc[j][2 * h + 1]);
                if (is_u) {   // U0 stored v-block major: [col/VB][i][col%VB]
                    *reinterpret_cast<float2*>(out + OFF_U0 + ((size_t)(col / VB) * C + i) * VB + (col % VB)) = v2;
                } else {
                    *reinterpret_cast<float2*>(out + OFF_X + (size_t)i * SA + col) = v2;
                }
            }
        }
    }
}

// ---------------------------------------------------------------------------
// inter-chunk recurrence: one CTA (4 warps) per (VB-row block of S, local v head).
// Chunk operands stream into shared memory with 1-D bulk async copies in two
// groups (A = X and the U0 slice, B = P and Kd), each refilled for the next
// chunk as soon as the current chunk has finished with it.
//   step 1 (all warps, 32 rows each):  [W; Q e^G] S^T  -> U (rows 0..63), Yp (64..127)
//   step 2 (warps 2, 3):              Y = Yp + P U
//   step 3 (all warps, 32 columns each): S = e^{G_last} S + U^T Kd
// ---------------------------------------------------------------------------
namespace gp {
constexpr int SU = VB + 8;   // U rows: conflict-free as row-major B and as transposed A
constexpr int NT1 = VB / 8;  // n-tiles of step 1 / 2
}
struct InterSmem {
    float X[2 * gp::C][gp::SA];   // [W; Q e^G]
    float Kd[gp::C][gp::SB];
    float P[gp::C][gp::SP];
    float U0[gp::C][gp::VB];
    float S[gp::VB][gp::SA];      // state rows [v][k]
    float U[gp::C][gp::SU];
    uint64_t barA, barB;
};

__device__ __forceinline__ void inter_issue_A(InterSmem& sm, const float* R, int vb, int lane) {
    using namespace gp;
    if (lane == 0) {
        mbar_arrive_expect_tx(&sm.barA, 2 * C * SA * 4 + C * VB * 4);
        bulk_g2s(&sm.X[0][0], R + OFF_X, 2 * C * SA * 4, &sm.barA);
        bulk_g2s(&sm.U0[0][0], R + OFF_U0 + (size_t)vb * C * VB, C * VB * 4, &sm.barA);
    }
}
__device__ __forceinline__ void inter_issue_B(InterSmem& sm, const float* R, int lane) {
    using namespace gp;
    if (lane == 0) {
        mbar_arrive_expect_tx(&sm.barB, C * SB * 4 + C * SP * 4);
        bulk_g2s(&sm.Kd[0][0], R + OFF_KD, C * SB * 4, &sm.barB);
        bulk_g2s(&sm.P[0][0], R + OFF_P, C * SP * 4, &sm.barB);
    }
}

__global__ void __launch_bounds__(128) gdn_pf_inter_kernel(int64_t T, int vc, const float* __restrict__ rec,
                                                           float* __restrict__ state, float* __restrict__ yraw,
                                                           int* err) {
    using namespace gp;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    InterSmem& sm = *reinterpret_cast<InterSmem*>(smem_raw);
    const int vb = blockIdx.x, vl = blockIdx.y, tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31, g = lane >> 2, t4 = lane & 3;
    float* Sg = state + ((size_t)vl * D + (size_t)vb * VB) * D;
    const int NC = (int)((T + C - 1) / C);
    if (tid == 0) {
        mbar_init(&sm.barA, 1);
        mbar_init(&sm.barB, 1);
        fence_mbar_init();
    }
    for (int i = tid; i < VB * (D / 4); i += 128) {
        const int r = i / (D / 4), c4 = i % (D / 4);
        *reinterpret_cast<float4*>(&sm.S[r][4 * c4]) = reinterpret_cast<const float4*>(Sg + (size_t)r * D)[c4];
    }
    __syncthreads();
    if (warp == 0) {
        const float* R0 = rec + (size_t)vl * REC;
        inter_issue_A(sm, R0, vb, lane);
        inter_issue_B(sm, R0, lane);
    }
    bool ok = true;
    for (int c = 0; c < NC; ++c) {
        const float* R = rec + ((size_t)c * vc + vl) * REC;
        const int64_t t0 = (int64_t)c * C;
        const int n = (int)(T - t0 < C ? T - t0 : C);
        // ---- step 1
        if (!mbar_wait(&sm.barA, (uint32_t)(c & 1), err)) ok = false;
        if (__syncthreads_or(!ok)) break;
        float acc[2][NT1][4];
#pragma unroll
        for (int mi = 0; mi < 2; ++mi)
#pragma unroll
            for (int j = 0; j < NT1; ++j)
#pragma unroll
                for (int e = 0; e < 4; ++e) acc[mi][j][e] = 0.0f;
        const int r0 = 32 * warp;
#pragma unroll 4
        for (int k0 = 0; k0 < D; k0 += 8) {
            FB bb[NT1];
#pragma unroll
            for (int j = 0; j < NT1; ++j) bb[j] = split_b(sm.S[8 * j + g][k0 + t4], sm.S[8 * j + g][k0 + t4 + 4]);
#pragma unroll
            for (int mi = 0; mi < 2; ++mi) {
                const int m0 = r0 + 16 * mi;
                const FA a = split_a(sm.X[m0 + g][k0 + t4], sm.X[m0 + g + 8][k0 + t4], sm.X[m0 + g][k0 + t4 + 4],
                                     sm.X[m0 + g + 8][k0 + t4 + 4]);
#pragma unroll
                for (int j = 0; j < NT1; ++j) mma3(acc[mi][j], a, bb[j]);
            }
        }
        if (warp < 2) {
#pragma unroll
            for (int mi = 0; mi < 2; ++mi)
#pragma unroll
                for (int j = 0; j < NT1; ++j)
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const int i = r0 + 16 * mi + g + (e >> 1) * 8;
                        const int v = 8 * j + 2 * t4 + (e & 1);
                        sm.U[i][v] = sm.U0[i][v] - acc[mi][j][e];
                    }
        }
        __syncthreads();                      // U complete; X, U0 free
        if (warp == 0 && c + 1 < NC) inter_issue_A(sm, R + (size_t)vc * REC, vb, lane);
        if (!mbar_wait(&sm.barB, (uint32_t)(c & 1), err)) ok = false;
        if (__syncthreads_or(!ok)) break;
        // ---- step 3 (every warp, columns 32w..32w+31): S_new = e^{G_last} S + U^T Kd
        float snew[4][4];
        {
            const float eGl = __ldg(R + OFF_EG);
            const int n0w = 32 * warp;
#pragma unroll
            for (int j = 0; j < 4; ++j)
#pragma unroll
                for (int e = 0; e < 4; ++e)
                    snew[j][e] = eGl * sm.S[g + (e >> 1) * 8][n0w + 8 * j + 2 * t4 + (e & 1)];
#pragma unroll 2
            for (int k0 = 0; k0 < C; k0 += 8) {
                const FA a = split_a(sm.U[k0 + t4][g], sm.U[k0 + t4][g + 8], sm.U[k0 + t4 + 4][g],
                                     sm.U[k0 + t4 + 4][g + 8]);
#pragma unroll
                for (int j = 0; j < 4; ++j)
                    mma3(snew[j], a, split_b(sm.Kd[k0 + t4][n0w + 8 * j + g], sm.Kd[k0 + t4 + 4][n0w + 8 * j + g]));
            }
        }
        // ---- step 2 (warps 2, 3): Y = Yp + P U
        if (warp >= 2) {
            const int yi0 = r0 - C;
#pragma unroll
            for (int mi = 0; mi < 2; ++mi) {
                const int m0 = yi0 + 16 * mi;
#pragma unroll 2
                for (int k0 = 0; k0 < C; k0 += 8) {
                    const FA a = split_a(sm.P[m0 + g][k0 + t4], sm.P[m0 + g + 8][k0 + t4], sm.P[m0 + g][k0 + t4 + 4],
                                         sm.P[m0 + g + 8][k0 + t4 + 4]);
#pragma unroll
                    for (int j = 0; j < NT1; ++j)
                        mma3(acc[mi][j], a, split_b(sm.U[k0 + t4][8 * j + g], sm.U[k0 + t4 + 4][8 * j + g]));
                }
#pragma unroll
                for (int j = 0; j < NT1; ++j)
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        const int i = m0 + g + 8 * h;
                        if (i < n) {
                            float* yo = yraw + ((size_t)(t0 + i) * vc + vl) * D + vb * VB + 8 * j + 2 * t4;
                            *reinterpret_cast<float2*>(yo) = make_float2(acc[mi][j][2 * h], acc[mi][j][2 * h + 1]);
                        }
                    }
            }
        }
        __syncthreads();                      // every read of S, U, P, Kd for this chunk is done
        {
            const int n0w = 32 * warp;
#pragma unroll
            for (int j = 0; j < 4; ++j)
#pragma unroll
                for (int h = 0; h < 2; ++h)
                    *reinterpret_cast<float2*>(&sm.S[g + 8 * h][n0w + 8 * j + 2 * t4]) =
                        make_float2(snew[j][2 * h], snew[j][2 * h + 1]);
        }
        if (warp == 0 && c + 1 < NC) inter_issue_B(sm, R + (size_t)vc * REC, lane);
        __syncthreads();
    }
    if (!ok) return;
    for (int i = tid; i < VB * (D / 4); i += 128) {
        const int r = i / (D / 4), c4 = i % (D / 4);
        reinterpret_cast<float4*>(Sg + (size_t)r * D)[c4] = *reinterpret_cast<const float4*>(&sm.S[r][4 * c4]);
    }
}

// ---------------------------------------------------------------------------
// gated RMSNorm (prefill variant, ss / head_dim; ssm.rs:294-334), per token
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) gdn_pf_gate_kernel(int vh0, int vc, const float* __restrict__ yraw,
                                                          const float* __restrict__ z,
                                                          const float* __restrict__ norm_w,
                                                          float* __restrict__ y_out) {
    const int64_t t = blockIdx.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const float4 w = reinterpret_cast<const float4*>(norm_w)[lane];
    for (int vl = warp; vl < vc; vl += 8) {
        const float4 y = reinterpret_cast<const float4*>(yraw + ((size_t)t * vc + vl) * SSM_D)[lane];
        const float ss = warp_sum(y.x * y.x + y.y * y.y + y.z * y.z + y.w * y.w);
        const float inv = 1.0f / sqrtf(ss / (float)SSM_D + 1e-6f);
        const float4 zz = reinterpret_cast<const float4*>(z + (size_t)t * INNER + (size_t)(vh0 + vl) * SSM_D)[lane];
        float4 o;
        o.x = ((y.x * inv) * w.x) * siluf_acc(zz.x);
        o.y = ((y.y * inv) * w.y) * siluf_acc(zz.y);
        o.z = ((y.z * inv) * w.z) * siluf_acc(zz.z);
        o.w = ((y.w * inv) * w.w) * siluf_acc(zz.w);
        reinterpret_cast<float4*>(y_out + ((size_t)t * vc + vl) * SSM_D)[lane] = o;
    }
}

cudaError_t launch_gdn_prefill(dz_ctx* ctx, int layer, int seq, int64_t T, const float* qkv, const float* alpha,
                               const float* beta, const float* z, float* y, cudaStream_t st, int* n_launch) {
    using namespace gp;
    const LayerState& L = ctx->layers[layer];
    const int vh0 = ctx->cfg.v_head_begin, vc = ctx->cfg.v_head_count;
    const SsmSlot slot = L.h_ssm[seq];
    const int h0 = L.head[seq];
    const int NC = (int)((T + C - 1) / C);
    const size_t n_qk = (size_t)T * SSM_HK * D, n_v = (size_t)T * vc * D, n_g = (size_t)T * vc;
    const size_t n_rec = (size_t)NC * vc * REC;
    const size_t total = 2 * n_qk + 2 * n_v + 2 * n_g + n_rec + 64;
    cudaError_t e = ensure_prefill_scratch(ctx, total * sizeof(float));
    if (e != cudaSuccess) return e;
    float* qn = static_cast<float*>(ctx->pf);
    float* kn = qn + n_qk;
    float* vv = kn + n_qk;
    float* yraw = vv + n_v;
    float* gl = yraw + n_v;
    float* bt = gl + n_g;
    float* rec = bt + n_g;
    rec = reinterpret_cast<float*>((reinterpret_cast<uintptr_t>(rec) + 15) & ~uintptr_t(15));

    gdn_pf_conv_kernel<<<(unsigned)T, 256, 0, st>>>(T, vh0, vc, h0, qkv, slot.hist, L.conv_w, L.ssm_a, L.dt_bias,
                                                    alpha, beta, qn, kn, vv, gl, bt);
    gdn_pf_ring_kernel<<<(unsigned)(T < CONV_K ? T : CONV_K), 256, 0, st>>>(T, h0, qkv, slot.hist);
    cudaFuncSetAttribute(gdn_pf_intra_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(IntraSmem));
    gdn_pf_intra_kernel<<<dim3(NC, vc), 256, sizeof(IntraSmem), st>>>(T, vh0, vc, qn, kn, vv, gl, bt, rec);
    cudaFuncSetAttribute(gdn_pf_inter_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(InterSmem));
    gdn_pf_inter_kernel<<<dim3(D / VB, vc), 128, sizeof(InterSmem), st>>>(T, vc, rec, slot.state, yraw, ctx->d_err);
    gdn_pf_gate_kernel<<<(unsigned)T, 256, 0, st>>>(vh0, vc, yraw, z, L.norm_w, y);
    *n_launch += 5;
    return cudaGetLastError();
}

}  // namespace dz
