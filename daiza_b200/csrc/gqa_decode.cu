// gqa_decode.cu -- split-K flash-decoding for the gated GQA core (decode).
//
// Reference: Daiza-engine/src/model/attention.rs:90-203 (one token per
// sequence).  Three stream-ordered kernels:
//   1. gqa_prep     : per sequence -- deinterleave [Q_h|gate_h], QK-RMSNorm,
//                     partial RoPE (the reference's '+' sign, math/rope.rs:205-210)
//                     at pos = len, q *= 1/16, append K/V at slot len.
//   2. gqa_split    : per (sequence, split-K chunk, kv head), one warp each --
//                     the 6 grouped q heads attend over the chunk's cached
//                     positions.  K/V tiles of 8 positions stream HBM -> shared
//                     memory through 1-D bulk async copies (cp.async.bulk +
//                     mbarrier, 3 stages per warp); scores on the FP32 pipes
//                     with a warp-shuffle reduce-scatter, online softmax in
//                     log2 units, unnormalised partials out.
//   3. gqa_combine  : per (sequence, kv head) -- merge the chunks' (m, l, o),
//                     divide, multiply by sigmoid(gate).
// Memory bound: every cached K and V byte is read exactly once.
#include <algorithm>
#include <cstddef>

#include "dz_internal.h"

namespace dz {

constexpr int STAGES = 3;

// ---------------------------------------------------------------------------
// 1. prep: 8 warps, one head task per warp-iteration.  tasks [0, nq) are q heads,
//    [nq, nq+kvc) are kv heads.  Lane l holds dims [4l,4l+4) and [128+4l,128+4l+4).
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) gqa_prep_kernel(GqaDecodeDesc d, int kvc, const KvSlot* __restrict__ kv,
                                                       const float* __restrict__ q_norm,
                                                       const float* __restrict__ k_norm,
                                                       const float* __restrict__ rope,
                                                       const float* __restrict__ q_gate,
                                                       const float* __restrict__ k_in,
                                                       const float* __restrict__ v_in,
                                                       float* __restrict__ q_buf, float eps) {
    const int b = blockIdx.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int sid = d.sid[b];
    const int pos = d.len[b];                      // cache slot (kv_cache.rs:79-88)
    const int nq = GRP * kvc;
    const KvSlot slot = kv[sid];
    const float* cs = rope + (size_t)d.pos[b] * (2 * ROPE);   // RoPE row of ModelState::pos (forward.rs:230-238)
    for (int task = warp; task < nq + kvc; task += 8) {
        const float* src;
        const float* w;
        float* dst;
        float scale;
        if (task < nq) {
            src = q_gate + ((size_t)b * nq + task) * QG_ROW;
            w = q_norm;
            dst = q_buf + ((size_t)b * nq + task) * HD;
            scale = 0.0625f;                     // 1/sqrt(256), attention.rs:110
        } else {
            const int h = task - nq;
            src = k_in + ((size_t)b * kvc + h) * HD;
            w = k_norm;
            dst = slot.k + ((size_t)h * slot.cap + pos) * HD;
            scale = 1.0f;
            // V is appended unchanged (kv_cache.rs:79-88)
            const float* vs = v_in + ((size_t)b * kvc + h) * HD;
            float* vd = slot.v + ((size_t)h * slot.cap + pos) * HD;
            reinterpret_cast<float4*>(vd)[lane] = reinterpret_cast<const float4*>(vs)[lane];
            reinterpret_cast<float4*>(vd)[lane + 32] = reinterpret_cast<const float4*>(vs)[lane + 32];
        }
        float4 x0 = reinterpret_cast<const float4*>(src)[lane];
        float4 x1 = reinterpret_cast<const float4*>(src)[lane + 32];
        float ss = x0.x * x0.x + x0.y * x0.y + x0.z * x0.z + x0.w * x0.w +
                   x1.x * x1.x + x1.y * x1.y + x1.z * x1.z + x1.w * x1.w;
        ss = warp_sum(ss);
        const float inv = 1.0f / sqrtf(ss / (float)HD + eps);     // rmsnorm.rs:284
        const float4 w0 = reinterpret_cast<const float4*>(w)[lane];
        const float4 w1 = reinterpret_cast<const float4*>(w)[lane + 32];
        x0 = make_float4((x0.x * inv) * w0.x, (x0.y * inv) * w0.y, (x0.z * inv) * w0.z, (x0.w * inv) * w0.w);
        x1 = make_float4((x1.x * inv) * w1.x, (x1.y * inv) * w1.y, (x1.z * inv) * w1.z, (x1.w * inv) * w1.w);
        // partial RoPE on dims [0,64): lanes 0..15 hold them; partner of dim i is i^32 (lane ^ 8)
        float4 pr;
        pr.x = __shfl_xor_sync(0xffffffffu, x0.x, 8);
        pr.y = __shfl_xor_sync(0xffffffffu, x0.y, 8);
        pr.z = __shfl_xor_sync(0xffffffffu, x0.z, 8);
        pr.w = __shfl_xor_sync(0xffffffffu, x0.w, 8);
        if (lane < 16) {
            const float4 c = reinterpret_cast<const float4*>(cs)[lane];          // cos[i] == cos[i^32]
            const float4 s = reinterpret_cast<const float4*>(cs + ROPE)[lane];
            // out = x*c + partner*s   (both halves use '+', math/rope.rs:205-210)
            x0 = make_float4(fmaf(x0.x, c.x, pr.x * s.x), fmaf(x0.y, c.y, pr.y * s.y),
                             fmaf(x0.z, c.z, pr.z * s.z), fmaf(x0.w, c.w, pr.w * s.w));
        }
        if (scale != 1.0f) {
            x0 = make_float4(x0.x * scale, x0.y * scale, x0.z * scale, x0.w * scale);
            x1 = make_float4(x1.x * scale, x1.y * scale, x1.z * scale, x1.w * scale);
        }
        reinterpret_cast<float4*>(dst)[lane] = x0;
        reinterpret_cast<float4*>(dst)[lane + 32] = x1;
    }
}

// ---------------------------------------------------------------------------
// 2. split-K attention, one WARP per work item (sequence, chunk, kv head).
//    Persistent CTAs of 4 independent warps (one CTA per SM).  Each warp walks
//    its own items and keeps its own ring of STAGES tiles of 8 positions in
//    shared memory, refilled by its lane 0 with two 1-D bulk async copies per
//    tile (K rows and V rows are each one contiguous run), across item
//    boundaries.  No CTA-wide barrier after set-up.
//    Lane l owns dims [4l,4l+4) and [128+4l,128+4l+4) of q (6 heads, in
//    registers), K, V and the output accumulators.
//    QK: 48 partial dot products per lane (8 positions x 6 heads), combined by
//        a 5-level reduce-scatter (48 shuffles per tile).
//    softmax: lanes 0..5 own heads (running max in log2 units, sum).
//    PV: every lane accumulates its 8 dims x 6 heads.
// ---------------------------------------------------------------------------
constexpr int TP = 8;        // positions per tile
constexpr int NWARP = 4;     // warps per CTA

// alignas(128): every warp's ring (and its K/V tiles, the bulk-copy
// destinations) must start on a 16-byte boundary, so the struct size must be a
// multiple of 16 -- the trailing mbarriers alone would only give 8.
struct alignas(128) WarpRing {
    float k[STAGES][TP][HD];
    float v[STAGES][TP][HD];
    float sc[TP][8];          // scores [pos][head] (log2 units)
    float p[TP][8];           // probabilities [pos][head]
    float alpha[8];
    uint64_t full[STAGES];
};
struct SplitSmem {
    WarpRing w[NWARP];
};
static_assert(sizeof(WarpRing) % 128 == 0, "per-warp rings must stay 16-byte aligned");
static_assert(offsetof(WarpRing, v) % 16 == 0 && offsetof(WarpRing, p) % 16 == 0 &&
              offsetof(WarpRing, alpha) % 16 == 0, "vector-loaded fields must be 16-byte aligned");

struct ItemInfo {
    int b, kvh, p0, p1, ntiles;
    const float* kb;
    const float* vb;
};

__device__ __forceinline__ ItemInfo decode_item(const GqaDecodeDesc& d, int kvc, const KvSlot* __restrict__ kv,
                                                int item) {
    ItemInfo it;
    const int chunk_idx = item / kvc;
    it.kvh = item - chunk_idx * kvc;
    int lo = 0, hi = d.B - 1;                    // last b with cum[b] <= chunk_idx
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (d.cum[mid] <= chunk_idx) lo = mid; else hi = mid - 1;
    }
    it.b = lo;
    const int c = chunk_idx - d.cum[lo];
    const int n = d.len[lo] + 1;
    it.p0 = c * d.chunk;
    it.p1 = min(n, it.p0 + d.chunk);
    it.ntiles = (it.p1 - it.p0 + TP - 1) / TP;
    const KvSlot slot = kv[d.sid[lo]];
    it.kb = slot.k + ((size_t)it.kvh * slot.cap + it.p0) * HD;
    it.vb = slot.v + ((size_t)it.kvh * slot.cap + it.p0) * HD;
    return it;
}

// keep the half of `in` selected by `hi` and add the partner lane's other half
template <int N>
__device__ __forceinline__ void rs_level(const float (&in)[2 * N], float (&out)[N], bool hi, int mask) {
#pragma unroll
    for (int i = 0; i < N; ++i) {
        const float send = hi ? in[i] : in[N + i];
        const float keep = hi ? in[N + i] : in[i];
        out[i] = keep + __shfl_xor_sync(0xffffffffu, send, mask);
    }
}

__global__ void __launch_bounds__(128, 1) gqa_split_kernel(GqaDecodeDesc d, int kvc, const KvSlot* __restrict__ kv,
                                                           const float* __restrict__ q_buf,
                                                           float* __restrict__ part_o,
                                                           float* __restrict__ part_ml, int* err, int n_items) {
    extern __shared__ __align__(128) unsigned char smem_raw[];
    SplitSmem& smem = *reinterpret_cast<SplitSmem*>(smem_raw);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    WarpRing& R = smem.w[warp];
    const int gw = blockIdx.x * NWARP + warp;
    const int nw = gridDim.x * NWARP;

    if (lane == 0) {
        for (int s = 0; s < STAGES; ++s) mbar_init(&R.full[s], 1);
        fence_mbar_init();
    }
    __syncwarp();

    // producer cursor (lane 0 issues, all lanes track it uniformly)
    int p_item = gw, p_tile = 0;
    ItemInfo pinfo{};
    if (p_item < n_items) pinfo = decode_item(d, kvc, kv, p_item);
    auto produce = [&](int stage) {
        if (p_item >= n_items) return;
        const int rows = min(TP, pinfo.p1 - (pinfo.p0 + p_tile * TP));
        if (lane == 0) {
            mbar_arrive_expect_tx(&R.full[stage], (uint32_t)rows * HD * 4 * 2);
            bulk_g2s(&R.k[stage][0][0], pinfo.kb + (size_t)p_tile * TP * HD, (uint32_t)rows * HD * 4, &R.full[stage]);
            bulk_g2s(&R.v[stage][0][0], pinfo.vb + (size_t)p_tile * TP * HD, (uint32_t)rows * HD * 4, &R.full[stage]);
        }
        if (++p_tile == pinfo.ntiles) {
            p_item += nw;
            p_tile = 0;
            if (p_item < n_items) pinfo = decode_item(d, kvc, kv, p_item);
        }
    };
    for (int s = 0; s < STAGES; ++s) produce(s);

    const int k_grp = lane >> 1;              // reduce-scatter group: indices 3k..3k+2 of (pos*6 + head)
    const int my_pos = k_grp >> 1;
    const int my_h0 = 3 * (k_grp & 1);
    const bool b4 = lane & 16, b3 = lane & 8, b2 = lane & 4, b1 = lane & 2;
    int j = 0;
    for (int item = gw; item < n_items; item += nw) {
        const ItemInfo it = decode_item(d, kvc, kv, item);
        float4 q[GRP][2];
        {
            const float* qs = q_buf + ((size_t)it.b * GRP * kvc + (size_t)it.kvh * GRP) * HD;
#pragma unroll
            for (int h = 0; h < GRP; ++h) {
                q[h][0] = *reinterpret_cast<const float4*>(qs + h * HD + 4 * lane);
                q[h][1] = *reinterpret_cast<const float4*>(qs + h * HD + 128 + 4 * lane);
            }
        }
        float o[GRP][8];
#pragma unroll
        for (int h = 0; h < GRP; ++h)
#pragma unroll
            for (int e = 0; e < 8; ++e) o[h][e] = 0.0f;
        float m_run = -INFINITY, l_run = 0.0f;     // meaningful in lanes 0..5 (head = lane)

        for (int t = 0; t < it.ntiles; ++t, ++j) {
            const int stage = j % STAGES;
            const int rows = min(TP, it.p1 - (it.p0 + t * TP));
            if (!mbar_wait(&R.full[stage], (uint32_t)((j / STAGES) & 1), err)) return;
            // ---- partial scores: part[p*6 + h] over this lane's 8 dims
            float part[TP * GRP];
#pragma unroll
            for (int p = 0; p < TP; ++p) {
                const float4 k0 = *reinterpret_cast<const float4*>(&R.k[stage][p][4 * lane]);
                const float4 k1 = *reinterpret_cast<const float4*>(&R.k[stage][p][128 + 4 * lane]);
#pragma unroll
                for (int h = 0; h < GRP; ++h) {
                    float a = k0.x * q[h][0].x;
                    a = fmaf(k0.y, q[h][0].y, a);
                    a = fmaf(k0.z, q[h][0].z, a);
                    a = fmaf(k0.w, q[h][0].w, a);
                    a = fmaf(k1.x, q[h][1].x, a);
                    a = fmaf(k1.y, q[h][1].y, a);
                    a = fmaf(k1.z, q[h][1].z, a);
                    a = fmaf(k1.w, q[h][1].w, a);
                    part[p * GRP + h] = a;
                }
            }
            // ---- reduce-scatter 48 -> 3 per lane pair (indices 3*k_grp .. 3*k_grp+2)
            float r24[24], r12[12], r6[6], r3[3];
            rs_level<24>(part, r24, b4, 16);
            rs_level<12>(r24, r12, b3, 8);
            rs_level<6>(r12, r6, b2, 4);
            rs_level<3>(r6, r3, b1, 2);
#pragma unroll
            for (int i = 0; i < 3; ++i) r3[i] += __shfl_xor_sync(0xffffffffu, r3[i], 1);
            if ((lane & 1) == 0) {
#pragma unroll
                for (int i = 0; i < 3; ++i) R.sc[my_pos][my_h0 + i] = r3[i] * LOG2E;
            }
            __syncwarp();
            // ---- online softmax: lane h < 6 owns head h
            if (lane < GRP) {
                float s[TP];
                float tmax = -INFINITY;
#pragma unroll
                for (int p = 0; p < TP; ++p) {
                    s[p] = p < rows ? R.sc[p][lane] : -INFINITY;
                    tmax = fmaxf(tmax, s[p]);
                }
                const float m_new = fmaxf(m_run, tmax);
                const float alpha = exp2f(m_run - m_new);
                float psum = 0.0f;
#pragma unroll
                for (int p = 0; p < TP; ++p) {
                    const float pe = p < rows ? exp2f(s[p] - m_new) : 0.0f;
                    R.p[p][lane] = pe;
                    psum += pe;
                }
                l_run = l_run * alpha + psum;
                m_run = m_new;
                R.alpha[lane] = alpha;
            }
            __syncwarp();
            // ---- o = alpha * o + P V
            {
                const float4 a03 = *reinterpret_cast<const float4*>(&R.alpha[0]);
                const float2 a45 = *reinterpret_cast<const float2*>(&R.alpha[4]);
                const float a[GRP] = {a03.x, a03.y, a03.z, a03.w, a45.x, a45.y};
                if (a[0] != 1.0f || a[1] != 1.0f || a[2] != 1.0f || a[3] != 1.0f || a[4] != 1.0f || a[5] != 1.0f) {
#pragma unroll
                    for (int h = 0; h < GRP; ++h)
#pragma unroll
                        for (int e = 0; e < 8; ++e) o[h][e] *= a[h];
                }
#pragma unroll
                for (int p = 0; p < TP; ++p) {
                    if (p < rows) {
                        const float4 pa = *reinterpret_cast<const float4*>(&R.p[p][0]);
                        const float2 pb = *reinterpret_cast<const float2*>(&R.p[p][4]);
                        const float pp[GRP] = {pa.x, pa.y, pa.z, pa.w, pb.x, pb.y};
                        const float4 v0 = *reinterpret_cast<const float4*>(&R.v[stage][p][4 * lane]);
                        const float4 v1 = *reinterpret_cast<const float4*>(&R.v[stage][p][128 + 4 * lane]);
                        const float vv[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
#pragma unroll
                        for (int h = 0; h < GRP; ++h)
#pragma unroll
                            for (int e = 0; e < 8; ++e) o[h][e] = fmaf(pp[h], vv[e], o[h][e]);
                    }
                }
            }
            __syncwarp();
            produce(stage);
        }
        // ---- write this item's unnormalised partial
        float* po = part_o + (size_t)item * GRP * HD;
#pragma unroll
        for (int h = 0; h < GRP; ++h) {
            *reinterpret_cast<float4*>(po + h * HD + 4 * lane) = make_float4(o[h][0], o[h][1], o[h][2], o[h][3]);
            *reinterpret_cast<float4*>(po + h * HD + 128 + 4 * lane) = make_float4(o[h][4], o[h][5], o[h][6], o[h][7]);
        }
        if (lane < GRP) {
            part_ml[((size_t)item * GRP + lane) * 2 + 0] = m_run;
            part_ml[((size_t)item * GRP + lane) * 2 + 1] = l_run;
        }
    }
}

// ---------------------------------------------------------------------------
// 3. combine chunks, normalise, gate.  grid (kvc, B), 256 threads (one dim each)
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) gqa_combine_kernel(GqaDecodeDesc d, int kvc, const float* __restrict__ part_o,
                                                          const float* __restrict__ part_ml,
                                                          const float* __restrict__ q_gate,
                                                          float* __restrict__ out) {
    __shared__ float wgt[MAXC][GRP];
    __shared__ float invl[GRP];
    const int kvh = blockIdx.x, b = blockIdx.y, tid = threadIdx.x;
    const int c0 = d.cum[b], nc = d.cum[b + 1] - d.cum[b];
    if (tid < GRP) {
        float M = -INFINITY;
        for (int c = 0; c < nc; ++c)
            M = fmaxf(M, part_ml[(((size_t)(c0 + c) * kvc + kvh) * GRP + tid) * 2]);
        float L = 0.0f;
        for (int c = 0; c < nc; ++c) {
            const size_t it = ((size_t)(c0 + c) * kvc + kvh) * GRP + tid;
            const float w = exp2f(part_ml[it * 2] - M);
            wgt[c][tid] = w;
            L = fmaf(part_ml[it * 2 + 1], w, L);
        }
        invl[tid] = 1.0f / L;
    }
    __syncthreads();
    const int nq = GRP * kvc;
#pragma unroll
    for (int h = 0; h < GRP; ++h) {
        float acc = 0.0f;
        for (int c = 0; c < nc; ++c)
            acc = fmaf(part_o[((size_t)(c0 + c) * kvc + kvh) * GRP * HD + h * HD + tid], wgt[c][h], acc);
        const int qh = kvh * GRP + h;
        const float g = q_gate[((size_t)b * nq + qh) * QG_ROW + HD + tid];
        out[((size_t)b * nq + qh) * HD + tid] = acc * invl[h] * sigmoidf_acc(g);
    }
}

cudaError_t launch_gqa_decode(dz_ctx* ctx, int layer, const GqaDecodeDesc& d, const float* q_gate,
                              const float* k, const float* v, float* out, cudaStream_t st, int* n_launch) {
    const LayerState& L = ctx->layers[layer];
    const int kvc = ctx->cfg.kv_head_count;
    const int items = d.cum[d.B] * kvc;
    cudaFuncSetAttribute(gqa_split_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(SplitSmem));
    gqa_prep_kernel<<<d.B, 256, 0, st>>>(d, kvc, L.d_kv, L.q_norm, L.k_norm, ctx->rope, q_gate, k, v, ctx->q_buf,
                                         ctx->cfg.rms_eps);
    const int grid = std::min((items + NWARP - 1) / NWARP, ctx->n_sm);
    gqa_split_kernel<<<grid, 32 * NWARP, sizeof(SplitSmem), st>>>(d, kvc, L.d_kv, ctx->q_buf, ctx->part_o,
                                                                  ctx->part_ml, ctx->d_err, items);
    gqa_combine_kernel<<<dim3(kvc, d.B), 256, 0, st>>>(d, kvc, ctx->part_o, ctx->part_ml, q_gate, out);
    *n_launch += 3;
    return cudaGetLastError();
}

}  // namespace dz

namespace dz {
// Same three launches as launch_gqa_decode, with the split-K scratch supplied by
// the caller instead of taken from the context (used by the no-allocation entry
// point, whose scratch is a fixed device array).
cudaError_t launch_gqa_decode_scratch(dz_ctx* ctx, int layer, const GqaDecodeDesc& d, const float* q_gate,
                                      const float* k, const float* v, float* out, cudaStream_t st, int* n_launch,
                                      float* q_buf, float* part_o, float* part_ml) {
    const LayerState& L = ctx->layers[layer];
    const int kvc = ctx->cfg.kv_head_count;
    const int items = d.cum[d.B] * kvc;
    cudaFuncSetAttribute(gqa_split_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(SplitSmem));
    gqa_prep_kernel<<<d.B, 256, 0, st>>>(d, kvc, L.d_kv, L.q_norm, L.k_norm, ctx->rope, q_gate, k, v, q_buf,
                                         ctx->cfg.rms_eps);
    const int grid = std::min((items + NWARP - 1) / NWARP, ctx->n_sm);
    gqa_split_kernel<<<grid, 32 * NWARP, sizeof(SplitSmem), st>>>(d, kvc, L.d_kv, q_buf, part_o, part_ml,
                                                                  ctx->d_err, items);
    gqa_combine_kernel<<<dim3(kvc, d.B), 256, 0, st>>>(d, kvc, part_o, part_ml, q_gate, out);
    *n_launch += 3;
    return cudaGetLastError();
}
}  // namespace dz
