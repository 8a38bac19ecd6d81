// gqa_decode.cu -- split-K flash-decoding for the gated GQA core (decode).
//
// Reference: Daiza-engine/src/model/attention.rs:90-203 (one token per
// sequence).  Three stream-ordered kernels:
//   1. gqa_prep     : per sequence -- deinterleave [Q_h|gate_h], QK-RMSNorm,
//                     partial RoPE (the reference's '+' sign, math/rope.rs:205-210)
//                     at pos = len, q *= 1/16, append K/V at slot len.
//   2. gqa_split    : per (sequence, split-K chunk, kv head) -- the 6 grouped q
//                     heads attend over the chunk's cached positions.  K/V tiles
//                     of 16 positions stream HBM -> shared memory through 1-D
//                     bulk async copies (cp.async.bulk + mbarrier, 3 stages);
//                     scores on the FP32 pipes, online softmax in log2 units
//                     with warp-shuffle reductions, unnormalised partials out.
//   3. gqa_combine  : per (sequence, kv head) -- merge the chunks' (m, l, o),
//                     divide, multiply by sigmoid(gate).
// Memory bound: every cached K and V byte is read exactly once.
#include "dz_internal.h"

namespace dz {

constexpr int TILE = 16;      // positions per pipeline stage
constexpr int STAGES = 3;
constexpr int KPAD = 260;     // padded K row in shared memory (floats): conflict-free row-per-lane reads

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
    const int pos = d.len[b];
    const int nq = GRP * kvc;
    const KvSlot slot = kv[sid];
    const float* cs = rope + (size_t)pos * (2 * ROPE);
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
// 2. split-K attention over one chunk
// ---------------------------------------------------------------------------
struct SplitSmem {
    float q[GRP][HD];                 // 6 KB
    float k[STAGES][TILE][KPAD];      // padded rows
    float v[STAGES][TILE][HD];
    float red[4][TILE][8];            // per-warp partial scores [warp][pos][head]
    float p[TILE][8];                 // probabilities [pos][head]
    float m[8], l[8], alpha[8];
    uint64_t full[STAGES];
};

__device__ __forceinline__ void issue_tile(SplitSmem& sm, int stage, int rows, const float* kb, const float* vb,
                                           int lane) {
    if (lane == 0) mbar_arrive_expect_tx(&sm.full[stage], (uint32_t)rows * HD * 4 * 2);
    __syncwarp();
    if (lane < rows) bulk_g2s(&sm.k[stage][lane][0], kb + (size_t)lane * HD, HD * 4, &sm.full[stage]);
    if (lane == 31) bulk_g2s(&sm.v[stage][0][0], vb, (uint32_t)rows * HD * 4, &sm.full[stage]);
}

__global__ void __launch_bounds__(128, 2) gqa_split_kernel(GqaDecodeDesc d, int kvc, const KvSlot* __restrict__ kv,
                                                           const float* __restrict__ q_buf,
                                                           float* __restrict__ part_o,
                                                           float* __restrict__ part_ml, int* err) {
    extern __shared__ __align__(128) unsigned char smem_raw[];
    SplitSmem& sm = *reinterpret_cast<SplitSmem*>(smem_raw);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int item = blockIdx.x;
    const int chunk_idx = item / kvc;
    const int kvh = item - chunk_idx * kvc;
    // b = last index with cum[b] <= chunk_idx
    int lo = 0, hi = d.B - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (d.cum[mid] <= chunk_idx) lo = mid; else hi = mid - 1;
    }
    const int b = lo;
    const int c = chunk_idx - d.cum[b];
    const int n = d.len[b] + 1;
    const int p0 = c * d.chunk;
    const int p1 = min(n, p0 + d.chunk);
    const int ntiles = (p1 - p0 + TILE - 1) / TILE;
    const KvSlot slot = kv[d.sid[b]];
    const float* kbase = slot.k + ((size_t)kvh * slot.cap + p0) * HD;
    const float* vbase = slot.v + ((size_t)kvh * slot.cap + p0) * HD;

    if (tid == 0) {
        for (int s = 0; s < STAGES; ++s) mbar_init(&sm.full[s], 1);
        fence_mbar_init();
    }
    if (tid < 8) { sm.m[tid] = -INFINITY; sm.l[tid] = 0.0f; sm.alpha[tid] = 1.0f; }
    {
        const float4* qs = reinterpret_cast<const float4*>(q_buf + ((size_t)b * GRP * kvc + (size_t)kvh * GRP) * HD);
        float4* qd = reinterpret_cast<float4*>(&sm.q[0][0]);
        for (int i = tid; i < GRP * HD / 4; i += 128) qd[i] = qs[i];
    }
    __syncthreads();
    if (warp == 0) {
        for (int j = 0; j < STAGES && j < ntiles; ++j) {
            const int rows = min(TILE, p1 - (p0 + j * TILE));
            issue_tile(sm, j, rows, kbase + (size_t)j * TILE * HD, vbase + (size_t)j * TILE * HD, lane);
        }
    }

    // thread roles
    const int qp = tid & 15;          // QK: position within tile
    const int qg = tid >> 4;          // QK: dim group of 32
    float o[GRP][2];
#pragma unroll
    for (int h = 0; h < GRP; ++h) { o[h][0] = 0.0f; o[h][1] = 0.0f; }
    bool ok = true;

    for (int j = 0; j < ntiles; ++j) {
        const int stage = j % STAGES;
        const int rows = min(TILE, p1 - (p0 + j * TILE));
        if (!mbar_wait(&sm.full[stage], (uint32_t)((j / STAGES) & 1), err)) { ok = false; }
        if (__syncthreads_or(!ok)) { ok = false; break; }
        // ---- scores: thread (qp, qg) covers 32 dims of one position for 6 heads
        {
            float acc[GRP];
#pragma unroll
            for (int h = 0; h < GRP; ++h) acc[h] = 0.0f;
            const float* krow = &sm.k[stage][qp][qg * 32];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const float4 kk = *reinterpret_cast<const float4*>(krow + 4 * i);
#pragma unroll
                for (int h = 0; h < GRP; ++h) {
                    const float4 qq = *reinterpret_cast<const float4*>(&sm.q[h][qg * 32 + 4 * i]);
                    acc[h] = fmaf(kk.x, qq.x, acc[h]);
                    acc[h] = fmaf(kk.y, qq.y, acc[h]);
                    acc[h] = fmaf(kk.z, qq.z, acc[h]);
                    acc[h] = fmaf(kk.w, qq.w, acc[h]);
                }
            }
#pragma unroll
            for (int h = 0; h < GRP; ++h) acc[h] += __shfl_xor_sync(0xffffffffu, acc[h], 16);
            if (lane < 16) {
                float* r = &sm.red[warp][qp][0];
                *reinterpret_cast<float4*>(r) = make_float4(acc[0], acc[1], acc[2], acc[3]);
                *reinterpret_cast<float2*>(r + 4) = make_float2(acc[4], acc[5]);
            }
        }
        __syncthreads();
        // ---- online softmax (log2 units): threads 0..95 = (head h, position p)
        if (tid < GRP * TILE) {
            const int h = tid >> 4, p = tid & 15;
            const bool valid = p < rows;
            float s = (sm.red[0][p][h] + sm.red[1][p][h] + sm.red[2][p][h] + sm.red[3][p][h]) * LOG2E;
            s = valid ? s : -INFINITY;
            float tmax = s;
#pragma unroll
            for (int off = 8; off > 0; off >>= 1) tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, off));
            const float m_old = sm.m[h];
            const float m_new = fmaxf(m_old, tmax);
            const float alpha = exp2f(m_old - m_new);
            const float pe = valid ? exp2f(s - m_new) : 0.0f;
            float psum = pe;
#pragma unroll
            for (int off = 8; off > 0; off >>= 1) psum += __shfl_xor_sync(0xffffffffu, psum, off);
            sm.p[p][h] = pe;
            if (p == 0) {
                sm.m[h] = m_new;
                sm.l[h] = sm.l[h] * alpha + psum;
                sm.alpha[h] = alpha;
            }
        }
        __syncthreads();
        // ---- o = alpha*o + P V : thread owns dims 2*tid, 2*tid+1
        {
#pragma unroll
            for (int h = 0; h < GRP; ++h) {
                const float a = sm.alpha[h];
                o[h][0] *= a;
                o[h][1] *= a;
            }
            for (int p = 0; p < rows; ++p) {
                const float4 pa = *reinterpret_cast<const float4*>(&sm.p[p][0]);
                const float2 pb = *reinterpret_cast<const float2*>(&sm.p[p][4]);
                const float2 vv = *reinterpret_cast<const float2*>(&sm.v[stage][p][2 * tid]);
                const float pp[GRP] = {pa.x, pa.y, pa.z, pa.w, pb.x, pb.y};
#pragma unroll
                for (int h = 0; h < GRP; ++h) {
                    o[h][0] = fmaf(pp[h], vv.x, o[h][0]);
                    o[h][1] = fmaf(pp[h], vv.y, o[h][1]);
                }
            }
        }
        __syncthreads();
        if (warp == 0 && j + STAGES < ntiles) {
            const int jn = j + STAGES;
            const int rn = min(TILE, p1 - (p0 + jn * TILE));
            issue_tile(sm, stage, rn, kbase + (size_t)jn * TILE * HD, vbase + (size_t)jn * TILE * HD, lane);
        }
    }
    if (!ok) return;
    float* po = part_o + (size_t)item * GRP * HD;
#pragma unroll
    for (int h = 0; h < GRP; ++h)
        *reinterpret_cast<float2*>(po + h * HD + 2 * tid) = make_float2(o[h][0], o[h][1]);
    if (tid < GRP) {
        part_ml[((size_t)item * GRP + tid) * 2 + 0] = sm.m[tid];
        part_ml[((size_t)item * GRP + tid) * 2 + 1] = sm.l[tid];
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
    gqa_split_kernel<<<items, 128, sizeof(SplitSmem), st>>>(d, kvc, L.d_kv, ctx->q_buf, ctx->part_o, ctx->part_ml,
                                                            ctx->d_err);
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
    gqa_split_kernel<<<items, 128, sizeof(SplitSmem), st>>>(d, kvc, L.d_kv, q_buf, part_o, part_ml, ctx->d_err);
    gqa_combine_kernel<<<dim3(kvc, d.B), 256, 0, st>>>(d, kvc, part_o, part_ml, q_gate, out);
    *n_launch += 3;
    return cudaGetLastError();
}
}  // namespace dz
