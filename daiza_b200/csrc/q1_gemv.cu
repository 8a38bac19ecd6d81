// q1_gemv.cu -- Q1_0 projection GEMV for a few tokens.
//
// Reference: Daiza-engine/src/model/weights.rs:831 (matvec_multi_into_slice: up
// to 8 Q1_0 matrices sharing one input row) with the row kernel
// tensor/quant.rs:267-328 (dot_q1_0_row_avx2) and its multi-token twin
// (weights.rs verify4t path).  Q1_0 row layout: cols/128 blocks of 18 bytes --
// the group scale as IEEE binary16 (little endian), then 16 sign bytes whose bit
// b of byte j is weight 8j + b (1 -> +scale, 0 -> -scale).
//
// With s_i = +-1 the signs of a group, sum_i s_i x_i = 2 sum_{bit_i = 1} x_i - sum_i x_i,
// and both sums are exact in integers once x is in fixed point:
//   1. q1_prep (one warp per (token, group of 128 inputs)): x ~= s_tg q with
//      |q| <= QMAX and s_tg = max|x over the group| / QMAX; q is stored as
//      three signed int8 digit planes (q = 65536 d2 + 256 d1 + d0) and, per
//      16-element slice, the sum of q (the "- sum x" term), in context-owned
//      scratch.
//   2. q1_gemv (one CTA of 16 warps per 64-row block of one matrix, a
//      programmatic dependent of 1): thread 0 starts the bulk copy of the
//      block's Q1_0 rows at once and the copy of the prepared input after the
//      grid-dependency wait.  Warp w takes rows 16 (w % 4) .. +15 over a quarter
//      of the groups (w / 4); a lane owns a 16-weight slice of each of its
//      groups for 4 rows, so each input slice it loads serves 4 rows: the
//      slice's 16 sign bits become four words of 0/1 bytes (one multiply and
//      one mask per 4 weights), __dp4a against the three digit planes gives the
//      integer sum over the set bits, 2 A - S the exact slice dot, and the
//      group scale (binary16 -> f32, exact) times s_tg weighs it into an f32
//      accumulator; shuffles sum the 8 slices of a row, shared memory the 4
//      quarters.
// The only rounding beyond f32 accumulation is the input quantisation (~1e-7 of
// the group's max|x| per element).  Roofline: HBM -- the Q1_0 bytes (1.125 bits
// per weight) are read once -- but the integer work per weight and token
// (4 ops to expand 4 signs, 12 dp4a per 16 weights) sets the pace.
#include <cuda_fp16.h>

#include <algorithm>
#include <cstddef>

#include "dz_internal.h"

namespace dz {

namespace q1 {
constexpr int ROWS = 64;         // rows per CTA: 4 row quads of 16 rows
constexpr int KSPLIT = 4;        // group quarters per row quad (one warp each)
constexpr int THREADS = 32 * 4 * KSPLIT;
constexpr int RL = 4;            // rows per lane: 4 row sets x 8 slices per warp, 4 rows per set
constexpr int PREP_WARPS = 8;    // groups per prep CTA
constexpr int QMAX = 8355000;    // |q| bound: three signed 8-bit digits reach +-8,355,711
constexpr int PLANES = 3;
}  // namespace q1

struct Q1Desc {
    int n_mats, cols, T;
    int accumulate;              // y += W x (matvec_add_into_slice) instead of y = W x
    const uint8_t* w[Q1_MAX_MATS];
    float* y[Q1_MAX_MATS];
    int rows[Q1_MAX_MATS];
    int blk0[Q1_MAX_MATS + 1];   // first CTA of each matrix
};

// prepared input (scratch, copied whole into each CTA's shared memory): digit planes
// [3][T][cols] int8 | slice sums [T][groups][8] int32 | group scales [T][groups] f32
// (padded to 16 bytes)
__host__ __device__ inline size_t q1_prep_bytes(int cols, int T) {
    const size_t groups = (size_t)cols / 128;
    return (size_t)q1::PLANES * T * cols + (size_t)T * groups * 8 * 4 + ((size_t)T * groups * 4 + 15) / 16 * 16;
}
size_t q1_smem_bytes(int cols, int T) {
    return (size_t)q1::ROWS * (cols / 128) * 18 + q1_prep_bytes(cols, T) + 32 +
           (size_t)q1::KSPLIT * q1::ROWS * T * 4;
}

// One (token t, group g) of the input -> fixed point, by one warp: lane l holds
// inputs 4l .. 4l+3 of the group (a 16-input slice is lanes 4k .. 4k+3).
__device__ __forceinline__ void quantise_group(float4 v, int t, int g, int groups, size_t plane, int cols, int lane,
                                               int8_t* planes, int* ssum, float* sxg) {
    using namespace q1;
    float mx = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
    mx = warp_max(mx);
    const float inv = mx > 0.0f ? (float)QMAX / mx : 0.0f;
    if (lane == 0) sxg[(size_t)t * groups + g] = mx > 0.0f ? mx / (float)QMAX : 0.0f;
    const float vv[4] = {v.x, v.y, v.z, v.w};
    uint32_t dw[PLANES] = {0u, 0u, 0u};
    int s4 = 0;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        int q = __float2int_rn(vv[e] * inv);
        q = max(-QMAX, min(QMAX, q));
        s4 += q;
#pragma unroll
        for (int p = 0; p < PLANES; ++p) {
            const int dgt = ((q + 128) & 255) - 128;   // digit in [-128, 127]
            dw[p] |= (uint32_t)(dgt & 0xFF) << (8 * e);
            q = (q - dgt) >> 8;                        // exact division
        }
    }
#pragma unroll
    for (int p = 0; p < PLANES; ++p)
        reinterpret_cast<uint32_t*>(planes + p * plane + (size_t)t * cols + (size_t)g * 128)[lane] = dw[p];
    s4 += __shfl_xor_sync(0xffffffffu, s4, 1);
    s4 += __shfl_xor_sync(0xffffffffu, s4, 2);
    if ((lane & 3) == 0) ssum[((size_t)t * groups + g) * 8 + (lane >> 2)] = s4;
}

// 1. grid (ceil(groups / 8), T): one warp per (token, group)
__global__ void __launch_bounds__(32 * q1::PREP_WARPS) q1_prep_kernel(const float* __restrict__ x, int cols, int T,
                                                                      unsigned char* __restrict__ prep) {
    using namespace q1;
    asm volatile("griddepcontrol.launch_dependents;");
    const int t = blockIdx.y, lane = threadIdx.x & 31;
    const int groups = cols / 128;
    const int g = blockIdx.x * PREP_WARPS + (threadIdx.x >> 5);
    if (g >= groups) return;
    const size_t plane = (size_t)T * cols;
    const float4 v = reinterpret_cast<const float4*>(x + (size_t)t * cols + (size_t)g * 128)[lane];
    quantise_group(v, t, g, groups, plane, cols, lane, reinterpret_cast<int8_t*>(prep),
                   reinterpret_cast<int*>(prep + PLANES * plane),
                   reinterpret_cast<float*>(prep + PLANES * plane + (size_t)T * groups * 8 * 4));
}

// ---------------------------------------------------------------------------
// 2. the GEMV
// ---------------------------------------------------------------------------
// TT: the launch's token count rounded up to 1, 2, 4 or 8 (register arrays sized by it)
template <int TT>
__global__ void __launch_bounds__(q1::THREADS, TT <= 2 ? 2 : 1) q1_gemv_kernel(Q1Desc d, const unsigned char* __restrict__ prep,
                                                                                 int* err) {
    using namespace q1;
    extern __shared__ __align__(128) unsigned char smem[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int cols = d.cols, T = d.T, groups = cols / 128;
    const int rowbytes = groups * 18;
    int m = 0;
    while ((int)blockIdx.x >= d.blk0[m + 1]) ++m;
    const int r0 = ((int)blockIdx.x - d.blk0[m]) * ROWS;
    const int nr = min(ROWS, d.rows[m] - r0);
    const size_t prep_bytes = q1_prep_bytes(cols, T);
    unsigned char* wsm = smem;
    unsigned char* psm = smem + (size_t)ROWS * rowbytes;
    const size_t plane = (size_t)T * cols;
    const int8_t* xd = reinterpret_cast<const int8_t*>(psm);
    const int* ssum = reinterpret_cast<const int*>(psm + PLANES * plane);
    const float* sxg = reinterpret_cast<const float*>(psm + PLANES * plane + (size_t)T * groups * 8 * 4);
    uint64_t* bar = reinterpret_cast<uint64_t*>(psm + prep_bytes);   // [2]: weights, prepared input
    float* part = reinterpret_cast<float*>(psm + prep_bytes + 32);    // [KSPLIT][ROWS][T] group-quarter sums

    if (tid == 0) {
        mbar_init(&bar[0], 1);
        mbar_init(&bar[1], 1);
        fence_mbar_init();
        const uint32_t bytes = (uint32_t)nr * (uint32_t)rowbytes;
        mbar_arrive_expect_tx(&bar[0], bytes);
        bulk_g2s(wsm, d.w[m] + (size_t)r0 * rowbytes, bytes, &bar[0]);
        // the prepared input comes from q1_prep, this grid's programmatic predecessor
        asm volatile("griddepcontrol.wait;" ::: "memory");
        mbar_arrive_expect_tx(&bar[1], (uint32_t)prep_bytes);
        bulk_g2s(psm, prep, (uint32_t)prep_bytes, &bar[1]);
    }
    __syncthreads();   // barrier initialisation visible to every waiting thread
    const bool ok = mbar_wait(&bar[0], 0, err) && mbar_wait(&bar[1], 0, err);

    const int sl = lane & 7;                            // 16-weight slice of each group
    const int rb = (warp & 3) * 16 + (lane >> 3) * RL;  // this lane's first row (block-local)
    const int kq = warp >> 2;                           // group quarter
    const int g0 = groups * kq / KSPLIT, g1 = groups * (kq + 1) / KSPLIT;
    float acc[RL][TT];
#pragma unroll
    for (int r = 0; r < RL; ++r)
#pragma unroll
        for (int t = 0; t < TT; ++t) acc[r][t] = 0.0f;
    if (ok) {
        for (int g = g0; g < g1; ++g) {
            int wk[RL][4];
            float sc[RL];
#pragma unroll
            for (int r = 0; r < RL; ++r) {
                uint32_t bits = 0;
                sc[r] = 0.0f;
                if (rb + r < nr) {
                    const unsigned char* blk = wsm + (size_t)(rb + r) * rowbytes + (size_t)g * 18;
                    sc[r] = __half2float(__ushort_as_half(*reinterpret_cast<const unsigned short*>(blk)));
                    bits = *reinterpret_cast<const unsigned short*>(blk + 2 + 2 * sl);
                }
#pragma unroll
                for (int k = 0; k < 4; ++k)
                    wk[r][k] = (int)((((bits >> (4 * k)) & 0xFu) * 0x00204081u) & 0x01010101u);   // bit j -> byte j
            }
#pragma unroll
            for (int t = 0; t < TT; ++t) {
                if (TT == 1 || t < T) {
                    const size_t off = (size_t)t * cols + g * 128 + 16 * sl;
                    const int4 x0 = *reinterpret_cast<const int4*>(xd + off);
                    const int4 x1 = *reinterpret_cast<const int4*>(xd + plane + off);
                    const int4 x2 = *reinterpret_cast<const int4*>(xd + 2 * plane + off);
                    const int S = ssum[((size_t)t * groups + g) * 8 + sl];
                    const float xs = sxg[(size_t)t * groups + g];
#pragma unroll
                    for (int r = 0; r < RL; ++r) {
                        int a0 = __dp4a(wk[r][0], x0.x, 0);
                        a0 = __dp4a(wk[r][1], x0.y, a0);
                        a0 = __dp4a(wk[r][2], x0.z, a0);
                        a0 = __dp4a(wk[r][3], x0.w, a0);
                        int a1 = __dp4a(wk[r][0], x1.x, 0);
                        a1 = __dp4a(wk[r][1], x1.y, a1);
                        a1 = __dp4a(wk[r][2], x1.z, a1);
                        a1 = __dp4a(wk[r][3], x1.w, a1);
                        int a2 = __dp4a(wk[r][0], x2.x, 0);
                        a2 = __dp4a(wk[r][1], x2.y, a2);
                        a2 = __dp4a(wk[r][2], x2.z, a2);
                        a2 = __dp4a(wk[r][3], x2.w, a2);
                        // |sum over set bits| <= 16 * QMAX < 2^28: 2 A - S stays inside int32
                        const int A = (a2 * 256 + a1) * 256 + a0;
                        acc[r][t] = fmaf(sc[r] * xs, (float)(2 * A - S), acc[r][t]);
                    }
                }
            }
        }
    }
#pragma unroll
    for (int r = 0; r < RL; ++r)
#pragma unroll
        for (int t = 0; t < TT; ++t) {
            float v = acc[r][t];
            v += __shfl_xor_sync(0xffffffffu, v, 1);
            v += __shfl_xor_sync(0xffffffffu, v, 2);
            v += __shfl_xor_sync(0xffffffffu, v, 4);
            acc[r][t] = v;
        }
    if (sl == 0) {
#pragma unroll
        for (int r = 0; r < RL; ++r)
#pragma unroll
            for (int t = 0; t < TT; ++t)
                if (t < T) part[((size_t)kq * ROWS + rb + r) * T + t] = acc[r][t];
    }
    __syncthreads();
    if (ok) {
        const int rows = d.rows[m];
        for (int i = tid; i < nr * T; i += THREADS) {
            const int r = i / T, t = i - r * T;
            float v = part[(size_t)r * T + t];
#pragma unroll
            for (int k = 1; k < KSPLIT; ++k) v += part[((size_t)k * ROWS + r) * T + t];
            float* yp = d.y[m] + (size_t)t * rows + r0 + r;
            *yp = d.accumulate ? *yp + v : v;
        }
    }
}

cudaError_t launch_q1_gemv(dz_ctx* ctx, int n_mats, const uint8_t* const* w, const int32_t* rows, int cols, int T,
                           const float* x, float* const* y, bool accumulate, cudaStream_t st, int* n_launch) {
    cudaError_t e = ensure_q1_scratch(ctx, q1_prep_bytes(cols, T));
    if (e != cudaSuccess) return e;
    unsigned char* prep = static_cast<unsigned char*>(ctx->q1);
    Q1Desc d{};
    d.n_mats = n_mats;
    d.cols = cols;
    d.T = T;
    d.accumulate = accumulate ? 1 : 0;
    d.blk0[0] = 0;
    for (int m = 0; m < n_mats; ++m) {
        d.w[m] = w[m];
        d.y[m] = y[m];
        d.rows[m] = rows[m];
        d.blk0[m + 1] = d.blk0[m] + (rows[m] + q1::ROWS - 1) / q1::ROWS;
    }
    for (int m = n_mats; m < Q1_MAX_MATS; ++m) d.blk0[m + 1] = d.blk0[n_mats];
    const int smem = (int)q1_smem_bytes(cols, T);
    auto kern = T <= 1 ? q1_gemv_kernel<1> : T <= 2 ? q1_gemv_kernel<2> : T <= 4 ? q1_gemv_kernel<4> : q1_gemv_kernel<8>;
    if ((e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem)) != cudaSuccess) return e;
    q1_prep_kernel<<<dim3((cols / 128 + q1::PREP_WARPS - 1) / q1::PREP_WARPS, T), 32 * q1::PREP_WARPS, 0, st>>>(
        x, cols, T, prep);
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t lc{};
    lc.gridDim = dim3(d.blk0[n_mats]);
    lc.blockDim = dim3(q1::THREADS);
    lc.dynamicSmemBytes = smem;
    lc.stream = st;
    lc.attrs = at;
    lc.numAttrs = 1;
    e = cudaLaunchKernelEx(&lc, kern, d, (const unsigned char*)prep, ctx->d_err);
    if (e != cudaSuccess) return e;
    *n_launch += 2;
    return cudaGetLastError();
}

}  // namespace dz
