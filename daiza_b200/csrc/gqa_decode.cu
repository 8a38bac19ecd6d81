// gqa_decode.cu -- split-K flash-decoding for the gated GQA core (decode).
//
// Reference: Daiza-engine/src/model/attention.rs:90-203 (one token per
// sequence).  Three stream-ordered kernels:
//   1. gqa_prep     : per sequence and head -- deinterleave [Q_h|gate_h],
//                     QK-RMSNorm, partial RoPE (the reference's '+' sign,
//                     math/rope.rs:205-210), q *= 1/16 -> q_buf; append K/V at
//                     slot len.
//   2. gqa_split    : per (sequence, split-K chunk, kv head), one warp each --
//                     the 6 grouped q heads attend over the chunk's cached
//                     positions.  K/V tiles of 4 positions stream HBM -> shared
//                     memory through 1-D bulk async copies (cp.async.bulk +
//                     mbarrier, 2 stages per warp, 8 warps per SM); scores on the FP32 pipes
//                     with a warp-shuffle reduce-scatter, online softmax in
//                     log2 units, unnormalised partials out.  A programmatic
//                     dependent of 1: old K/V tiles stream in while 1 finishes.
//   3. gqa_combine  : per (q head, sequence), a programmatic dependent of 2 --
//                     merge the chunks' (m, l, o), divide, multiply by
//                     sigmoid(gate).
// Memory bound: every cached K and V byte is read exactly once.
#include <algorithm>
#include <cstddef>

#include "dz_internal.h"

namespace dz {

constexpr int STAGES = 2;

// ---------------------------------------------------------------------------
// Per-head prologue (attention.rs:92-113) on a loaded head row: RMSNorm
// (rmsnorm.rs:284, (x*inv)*w), partial RoPE on dims [0, 64) with the reference's
// '+' sign for both halves (math/rope.rs:205-210), then the scale (1/sqrt(256)
// for q, 1 for k).  One warp per head row of 256; lane l holds dims [4l,4l+4)
// (x0) and [128+4l,128+4l+4) (x1); c/sn are the RoPE cos/sin of dims [4l,4l+4)
// (lanes 0..15).  The partner of dim i < 32 is i + 32, i.e. lane ^ 8.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void norm_rope(float4& x0, float4& x1, const float4 w0, const float4 w1, const float4 c,
                                          const float4 sn, float eps, float scale, int lane) {
    float ss = x0.x * x0.x + x0.y * x0.y + x0.z * x0.z + x0.w * x0.w +
               x1.x * x1.x + x1.y * x1.y + x1.z * x1.z + x1.w * x1.w;
    ss = warp_sum(ss);
    const float inv = 1.0f / sqrtf(ss / (float)HD + eps);
    x0 = make_float4((x0.x * inv) * w0.x, (x0.y * inv) * w0.y, (x0.z * inv) * w0.z, (x0.w * inv) * w0.w);
    x1 = make_float4((x1.x * inv) * w1.x, (x1.y * inv) * w1.y, (x1.z * inv) * w1.z, (x1.w * inv) * w1.w);
    float4 pr;
    pr.x = __shfl_xor_sync(0xffffffffu, x0.x, 8);
    pr.y = __shfl_xor_sync(0xffffffffu, x0.y, 8);
    pr.z = __shfl_xor_sync(0xffffffffu, x0.z, 8);
    pr.w = __shfl_xor_sync(0xffffffffu, x0.w, 8);
    if (lane < 16)   // cos[i] == cos[i^32]; out = x*c + partner*s for both halves
        x0 = make_float4(fmaf(x0.x, c.x, pr.x * sn.x), fmaf(x0.y, c.y, pr.y * sn.y),
                         fmaf(x0.z, c.z, pr.z * sn.z), fmaf(x0.w, c.w, pr.w * sn.w));
    if (scale != 1.0f) {
        x0 = make_float4(x0.x * scale, x0.y * scale, x0.z * scale, x0.w * scale);
        x1 = make_float4(x1.x * scale, x1.y * scale, x1.z * scale, x1.w * scale);
    }
}

// ---------------------------------------------------------------------------
// 1. gqa_prep: grid (B, ceil((nq + kvc) / 8)), one head task per warp.  Tasks [0, nq) are q heads -> q_buf; [nq, nq + kvc) are kv
//    heads: K (normed, RoPE'd) and V appended at slot len (kv_cache.rs:79-88).
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) gqa_prep_kernel(GqaDecodeDesc d, int kvc, const KvSlot* __restrict__ kv,
                                                       const float* __restrict__ q_norm,
                                                       const float* __restrict__ k_norm,
                                                       const float* __restrict__ rope,
                                                       const float* __restrict__ q_gate,
                                                       const float* __restrict__ k_in,
                                                       const float* __restrict__ v_in,
                                                       float* __restrict__ q_buf, float eps) {
    // Launched as a programmatic dependent of whatever precedes it: wait for that
    // grid first (inputs, q_buf and the caches may still be in use by it), and only
    // then let the split grid launch -- the split grid streams old K/V tiles before
    // its own wait, so every earlier append must be complete by then.
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;");
    const int b = blockIdx.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nq = GRP * kvc;
    const int task = blockIdx.y * 8 + warp;
    if (task >= nq + kvc) return;
    const float* cs = rope + (size_t)d.pos[b] * (2 * ROPE);   // RoPE row of ModelState::pos (forward.rs:230-238)
    const float4 zero4 = make_float4(0.f, 0.f, 0.f, 0.f);
    const float4 rc = lane < 16 ? reinterpret_cast<const float4*>(cs)[lane] : zero4;
    const float4 rs = lane < 16 ? reinterpret_cast<const float4*>(cs + ROPE)[lane] : zero4;
    if (task < nq) {
        const float4* src = reinterpret_cast<const float4*>(q_gate + ((size_t)b * nq + task) * QG_ROW);
        float4 x0 = src[lane], x1 = src[lane + 32];
        norm_rope(x0, x1, reinterpret_cast<const float4*>(q_norm)[lane],
                  reinterpret_cast<const float4*>(q_norm)[lane + 32], rc, rs, eps, 0.0625f, lane);
        float4* dst = reinterpret_cast<float4*>(q_buf + ((size_t)b * nq + task) * HD);
        dst[lane] = x0;
        dst[lane + 32] = x1;
    } else {
        const int h = task - nq;
        const KvSlot slot = kv[d.sid[b]];
        const float4* ks = reinterpret_cast<const float4*>(k_in + ((size_t)b * kvc + h) * HD);
        const float4* vs = reinterpret_cast<const float4*>(v_in + ((size_t)b * kvc + h) * HD);
        float4 x0 = ks[lane], x1 = ks[lane + 32];
        const float4 v0 = vs[lane], v1 = vs[lane + 32];
        norm_rope(x0, x1, reinterpret_cast<const float4*>(k_norm)[lane],
                  reinterpret_cast<const float4*>(k_norm)[lane + 32], rc, rs, eps, 1.0f, lane);
        float4* kd = reinterpret_cast<float4*>(slot.k + ((size_t)h * slot.cap + d.len[b]) * HD);
        float4* vd = reinterpret_cast<float4*>(slot.v + ((size_t)h * slot.cap + d.len[b]) * HD);
        kd[lane] = x0;
        kd[lane + 32] = x1;
        vd[lane] = v0;
        vd[lane + 32] = v1;
    }
}

// ---------------------------------------------------------------------------
// 2. split-K attention, one WARP per work item (sequence, chunk, kv head).
//    Persistent CTAs of 8 independent warps (one CTA per SM, two warps per
//    sub-partition so one warp's stalls hide under the other's work).  Each
//    warp walks its own items and keeps its own ring of STAGES tiles of 4
//    positions in shared memory, refilled by its lane 0 with two 1-D bulk async
//    copies per tile (K rows and V rows are each one contiguous run), across
//    item boundaries.  No CTA-wide barrier after set-up.  (Measured on config 2:
//    8 warps x 2 stages x 4 positions 0.93 of HBM; 4 warps x 3 x 8 positions
//    0.85; 12 warps exceed the register file.)
//    Lane l owns dims [4l,4l+4) and [128+4l,128+4l+4) of q (6 heads, in
//    registers), K, V and the output accumulators.
//    QK: 24 partial dot products per lane (4 positions x 6 heads), combined by
//        a reduce-scatter over lane bits 16, 8, 4 and sums over bits 2, 1.
//    softmax: lanes 0..5 own heads (running max in log2 units, sum).
//    PV: every lane accumulates its 8 dims x 6 heads.
// ---------------------------------------------------------------------------
constexpr int TP = 4;        // positions per tile
constexpr int NWARP = GQA_SPLIT_WARPS;     // warps per CTA (8)

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

__global__ void __launch_bounds__(32 * NWARP, 1) gqa_split_kernel(GqaDecodeDesc d, int kvc, const KvSlot* __restrict__ kv,
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

    // the combine grid may launch now; it waits for this grid before reading partials
    asm volatile("griddepcontrol.launch_dependents;");
    // producer cursor (lane 0 issues, all lanes track it uniformly)
    int p_item = gw, p_tile = 0;
    ItemInfo pinfo{};
    if (p_item < n_items) pinfo = decode_item(d, kvc, kv, p_item);
    // gqa_prep (the programmatic predecessor) appends the row at slot len, so a
    // tile that holds it is requested only after the grid-dependency wait
    bool dep_done = false;
    auto wait_prep = [&]() {
        if (!dep_done) {
            asm volatile("griddepcontrol.wait;" ::: "memory");
            dep_done = true;
        }
    };
    auto produce = [&](int stage) {
        if (p_item >= n_items) return;
        const int rows = min(TP, pinfo.p1 - (pinfo.p0 + p_tile * TP));
        if (pinfo.p0 + p_tile * TP + rows > d.len[pinfo.b]) wait_prep();
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
    wait_prep();   // q_buf comes from gqa_prep

    const int k_grp = lane >> 2;              // reduce-scatter group: indices 3k..3k+2 of (pos*6 + head)
    const int my_pos = k_grp >> 1;
    const int my_h0 = 3 * (k_grp & 1);
    const bool b4 = lane & 16, b3 = lane & 8, b2 = lane & 4;
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
            // ---- reduce-scatter 24 -> 3 per lane quad (indices 3*k_grp .. 3*k_grp+2)
            float r12[12], r6[6], r3[3];
            rs_level<12>(part, r12, b4, 16);
            rs_level<6>(r12, r6, b3, 8);
            rs_level<3>(r6, r3, b2, 4);
#pragma unroll
            for (int i = 0; i < 3; ++i) {
                r3[i] += __shfl_xor_sync(0xffffffffu, r3[i], 2);
                r3[i] += __shfl_xor_sync(0xffffffffu, r3[i], 1);
            }
            if ((lane & 3) == 0) {
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
// 3. combine chunks, normalise, gate.  One CTA per (q head, sequence) of
//    32 * G threads (G = 8, 16 or 32 chunk groups, enough threads for one
//    (m, l) pair each): group g sums chunks g, g + G, ... with lane l owning
//    dims [4l,4l+4) and [128+4l,128+4l+4); the G group sums meet in shared
//    memory.  Launched as a programmatic dependent of the split grid.
// ---------------------------------------------------------------------------
constexpr int CMB_MAX_GROUPS = 32;
static_assert(MAXC <= 32 * CMB_MAX_GROUPS, "one (m, l) pair per thread");
__global__ void __launch_bounds__(32 * CMB_MAX_GROUPS) gqa_combine_kernel(GqaDecodeDesc d, int kvc,
                                                                          const float* __restrict__ part_o,
                                                                          const float* __restrict__ part_ml,
                                                                          const float* __restrict__ q_gate,
                                                                          float* __restrict__ out) {
    __shared__ float wgt[MAXC];
    __shared__ float red[2][CMB_MAX_GROUPS];
    // a programmatic successor (the next projection) may start streaming its weights
    asm volatile("griddepcontrol.launch_dependents;");
    __shared__ __align__(16) float acc_s[CMB_MAX_GROUPS][HD];
    const int nq = GRP * kvc;
    const int qh = blockIdx.x, b = blockIdx.y, tid = threadIdx.x;
    const int kvh = qh / GRP, h = qh - kvh * GRP;
    const int warp = tid >> 5, lane = tid & 31, groups = blockDim.x >> 5;
    // an input, readable before the grid-dependency wait
    const float gate = tid < HD ? q_gate[((size_t)b * nq + qh) * QG_ROW + HD + tid] : 0.0f;
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int c0 = d.cum[b], nc = d.cum[b + 1] - d.cum[b];   // nc <= blockDim.x
    float m = -INFINITY, l = 0.0f;
    if (tid < nc) {
        const float2 ml = *reinterpret_cast<const float2*>(part_ml + (((size_t)(c0 + tid) * kvc + kvh) * GRP + h) * 2);
        m = ml.x;
        l = ml.y;
    }
    const float wm = warp_max(m);
    if (lane == 0) red[0][warp] = wm;
    __syncthreads();
    float M = red[0][0];
    for (int w = 1; w < groups; ++w) M = fmaxf(M, red[0][w]);
    float lw = 0.0f;
    if (tid < nc) {
        const float w = exp2f(m - M);
        wgt[tid] = w;
        lw = l * w;
    }
    lw = warp_sum(lw);
    if (lane == 0) red[1][warp] = lw;
    __syncthreads();
    float4 a0 = make_float4(0.f, 0.f, 0.f, 0.f), a1 = a0;
    const float* base = part_o + (size_t)h * HD + 4 * lane;
#pragma unroll 4
    for (int c = warp; c < nc; c += groups) {
        const float* po = base + ((size_t)(c0 + c) * kvc + kvh) * GRP * HD;
        const float4 x0 = *reinterpret_cast<const float4*>(po);
        const float4 x1 = *reinterpret_cast<const float4*>(po + 128);
        const float w = wgt[c];
        a0.x = fmaf(x0.x, w, a0.x); a0.y = fmaf(x0.y, w, a0.y); a0.z = fmaf(x0.z, w, a0.z); a0.w = fmaf(x0.w, w, a0.w);
        a1.x = fmaf(x1.x, w, a1.x); a1.y = fmaf(x1.y, w, a1.y); a1.z = fmaf(x1.z, w, a1.z); a1.w = fmaf(x1.w, w, a1.w);
    }
    *reinterpret_cast<float4*>(&acc_s[warp][4 * lane]) = a0;
    *reinterpret_cast<float4*>(&acc_s[warp][128 + 4 * lane]) = a1;
    __syncthreads();
    if (tid < HD) {
        float L = 0.0f;
        for (int w = 0; w < groups; ++w) L += red[1][w];
        float o = 0.0f;
        for (int g = 0; g < groups; ++g) o += acc_s[g][tid];
        out[((size_t)b * nq + qh) * HD + tid] = o * (1.0f / L) * sigmoidf_acc(gate);
    }
}

// prep as a programmatic dependent of whatever came before in the stream (it
// waits for that grid before anything else), then the split grid as a
// programmatic dependent of prep (old K/V tiles stream in while prep finishes)
// and the combine grid as a programmatic dependent of split.
cudaError_t launch_gqa_decode_scratch(dz_ctx* ctx, int layer, const GqaDecodeDesc& d, const float* q_gate,
                                      const float* k, const float* v, float* out, cudaStream_t st, int* n_launch,
                                      float* q_buf, float* part_o, float* part_ml) {
    const LayerState& L = ctx->layers[layer];
    const int kvc = ctx->cfg.kv_head_count;
    const int items = d.cum[d.B] * kvc;
    int max_nc = 0;
    for (int b = 0; b < d.B; ++b) max_nc = std::max(max_nc, d.cum[b + 1] - d.cum[b]);
    cudaError_t e = cudaFuncSetAttribute(gqa_split_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)sizeof(SplitSmem));
    if (e != cudaSuccess) return e;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    {
        cudaLaunchConfig_t lp{};
        lp.gridDim = dim3(d.B, (GRP * kvc + kvc + 7) / 8);
        lp.blockDim = dim3(256);
        lp.stream = st;
        lp.attrs = at;
        lp.numAttrs = 1;
        e = cudaLaunchKernelEx(&lp, gqa_prep_kernel, d, kvc, (const KvSlot*)L.d_kv, (const float*)L.q_norm,
                               (const float*)L.k_norm, (const float*)ctx->rope, q_gate, k, v, q_buf,
                               ctx->cfg.rms_eps);
        if (e != cudaSuccess) return e;
    }
    cudaLaunchConfig_t lc{};
    lc.gridDim = dim3(std::min((items + NWARP - 1) / NWARP, ctx->n_sm));
    lc.blockDim = dim3(32 * NWARP);
    lc.dynamicSmemBytes = sizeof(SplitSmem);
    lc.stream = st;
    lc.attrs = at;
    lc.numAttrs = 1;
    e = cudaLaunchKernelEx(&lc, gqa_split_kernel, d, kvc, (const KvSlot*)L.d_kv, (const float*)q_buf, part_o,
                           part_ml, ctx->d_err, items);
    if (e != cudaSuccess) return e;
    const int groups = max_nc > 256 / 2 ? 32 : (max_nc > 64 ? 16 : 8);
    lc.gridDim = dim3(GRP * kvc, d.B);
    lc.blockDim = dim3(32 * groups);
    lc.dynamicSmemBytes = 0;
    e = cudaLaunchKernelEx(&lc, gqa_combine_kernel, d, kvc, (const float*)part_o, (const float*)part_ml, q_gate, out);
    if (e != cudaSuccess) return e;
    *n_launch += 3;
    return cudaGetLastError();
}

cudaError_t launch_gqa_decode(dz_ctx* ctx, int layer, const GqaDecodeDesc& d, const float* q_gate,
                              const float* k, const float* v, float* out, cudaStream_t st, int* n_launch) {
    return launch_gqa_decode_scratch(ctx, layer, d, q_gate, k, v, out, st, n_launch, ctx->q_buf, ctx->part_o,
                                     ctx->part_ml);
}

}  // namespace dz
