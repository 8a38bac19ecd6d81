// gqa_prefill.cu -- causal GQA prefill: TMA-fed tcgen05/TMEM flash attention.
//
// Reference: Daiza-engine/src/model/forward.rs:599-721 (parallel GQA prefill):
// K-norm + RoPE + append for every token first, then each token t attends over
// base_len + t + 1 cached positions with Q-norm/RoPE/scale applied to its q,
// and the output is multiplied by sigmoid(gate).
//
// Kernels (stream-ordered):
//   1. pf_prep      : per token -- QK-RMSNorm, partial RoPE ('+' sign), q *= 1/16;
//                     writes Q as bf16 [head][T][256], appends K (normed, roped) and
//                     V to the f32 KV cache and to bf16 copies [kvh][len][256].
//   2. pf_prior     : (only when the cache already held tokens) bf16 copies of the
//                     prior K/V rows for the attention kernel.
//   3. pf_attn      : one CTA per (q head, 128-token query tile), heaviest tiles
//                     first.  Warp 8 issues TMA loads (Q once; K blocks of 128 keys
//                     as 16 KB 64-dim boxes through a 5-slot ring, V as 16 KB
//                     32-key slots through a 4-slot ring, all 128B-swizzled), warp 9
//                     issues tcgen05.mma from a single thread: S = Q K^T (M128 N128
//                     K256, both operands K-major in SMEM) into one of two TMEM S
//                     buffers, and O += P V (M128 N256 K128, P from TMEM, V MN-major
//                     in SMEM) into a 256-column TMEM accumulator.  Warps 0-7 (one
//                     TMEM lane per query row, two warps per lane quarter splitting
//                     the 128 keys of a block) run the causal online softmax in log2 units
//                     with a lazy rescale of O (only when the row max grows by more
//                     than 2^8), write P as bf16 over its S columns in TMEM, and finish with
//                     O / l * sigmoid(gate).
// All mbarrier waits are bounded (device error word on expiry).
#include <cuda.h>
#include <cuda_bf16.h>
#include <cstddef>
#include <algorithm>

#include "dz_internal.h"

namespace dz {

namespace pf {

constexpr int BM = 128;        // query rows per CTA
constexpr int BN = 128;        // keys per block (S = Q K^T runs as M128 x N128 products)
constexpr int NK = 5;          // K ring: slots of one 64-dim box of a key block (128 x 64 bf16, 16 KB)
constexpr int NV = 4;          // V ring: slots of 32 keys x 256 dims (4 boxes of 32 x 64 bf16, 16 KB)
constexpr int NTHREADS = 320;  // warps 0-7 softmax, warp 8 TMA, warp 9 MMA
// TMEM columns: S buffers [0,128) and [128,256) (f32); P of a block (bf16 pairs)
// overwrites the first 64 columns of its own S buffer; O accumulator [256,512)
__host__ __device__ constexpr uint32_t S_COL(int st) { return 128u * (uint32_t)st; }
constexpr uint32_t O_COL = 256;
constexpr float RESCALE_THRESHOLD = 8.0f;   // log2 units

struct alignas(1024) Smem {
    __nv_bfloat16 q[4][BM][64];          // 4 boxes of 64 dims, 16 KB each
    __nv_bfloat16 k[NK][BN][64];         // K ring
    __nv_bfloat16 v[NV][4][32][64];      // V ring
    uint64_t q_full;
    uint64_t k_full[NK], k_empty[NK], v_full[NV], v_empty[NV];
    uint64_t s_full[2], p_full[2], pv_done[2];
    float red_max[2][2][BM];             // [block parity][column half][row] partial row maxima
    float red_l[2][BM];                  // [column half][row] partial row sums
    uint32_t tmem_base;
};
static_assert(offsetof(Smem, k) % 1024 == 0 && offsetof(Smem, v) % 1024 == 0, "swizzle atoms need 1 KB alignment");

// ---- PTX wrappers --------------------------------------------------------
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int c0, int c1, int c2, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];"
        ::"r"(smem_u32(dst)), "l"(map), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2) : "memory");
}
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
                 "r"(ncols) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void fence_before_sync() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after_sync() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
// D[tmem] (+)= A[smem desc] * B[smem desc]
__device__ __forceinline__ void umma_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                        uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate) : "memory");
}
// D[tmem] (+)= A[tmem] * B[smem desc]
__device__ __forceinline__ void umma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                        uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}"
        ::"r"(d_tmem), "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate) : "memory");
}
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float* v) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}
// 32 columns into registers without waiting (pair with tmem_wait_ld)
__device__ __forceinline__ void tmem_ld32_async(uint32_t taddr, uint32_t* r) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t* r) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};"
        ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
          "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]),
          "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]),
          "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t* r) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};"
        ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
          "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
        : "memory");
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}
// barrier among a subset of the CTA's warps (id 0 is __syncthreads)
__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// SMEM matrix descriptor, 128-byte swizzle (sm100 layout: version 1 at bit 46,
// layout type 2 at bits 61-63; addresses and offsets in 16-byte units).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
    return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)((lbo_bytes >> 4) & 0x3FFF) << 16) |
           ((uint64_t)((sbo_bytes >> 4) & 0x3FFF) << 32) | ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
// Instruction descriptor, kind::f16: bf16 A and B, f32 accumulator.
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N, bool b_mn_major) {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((b_mn_major ? 1u : 0u) << 16) | ((uint32_t)(N >> 3) << 17) |
           ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ bool wait_or_flag(uint64_t* bar, uint32_t parity, int* err, bool& ok) {
    if (!ok) return false;
    if (!mbar_wait(bar, parity, err)) ok = false;
    return ok;
}

__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// three-input maximum (sm_100)
__device__ __forceinline__ float max3f(float a, float b, float c) {
    float d;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}
// packed f32x2 arithmetic on register pairs (sm_100)
__device__ __forceinline__ uint64_t f2(float a, float b) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
    return r;
}
__device__ __forceinline__ void f2_split(uint64_t r, float& a, float& b) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(r));
}
__device__ __forceinline__ uint64_t sub_f2(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ uint64_t add_f2(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}

__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
    const __nv_bfloat162 v = __floats2bfloat162_rn(a, b);   // .x = a (low half)
    return *reinterpret_cast<const uint32_t*>(&v);
}

}  // namespace pf

// ---------------------------------------------------------------------------
// 1. prep: per token (blockIdx.x), 8 warps over 6*kvc q heads and kvc kv heads
// ---------------------------------------------------------------------------
template <typename Tin>
__device__ __forceinline__ float4 ld4(const Tin* p);
template <>
__device__ __forceinline__ float4 ld4<float>(const float* p) { return *reinterpret_cast<const float4*>(p); }
template <>
__device__ __forceinline__ float4 ld4<__nv_bfloat16>(const __nv_bfloat16* p) {
    const uint2 u = *reinterpret_cast<const uint2*>(p);
    const __nv_bfloat162 a = *reinterpret_cast<const __nv_bfloat162*>(&u.x);
    const __nv_bfloat162 b = *reinterpret_cast<const __nv_bfloat162*>(&u.y);
    return make_float4(__low2float(a), __high2float(a), __low2float(b), __high2float(b));
}
__device__ __forceinline__ void st4_bf16(__nv_bfloat16* p, float4 x) {
    uint2 u;
    u.x = pf::pack_bf16(x.x, x.y);
    u.y = pf::pack_bf16(x.z, x.w);
    *reinterpret_cast<uint2*>(p) = u;
}

template <typename Tin>
__global__ void __launch_bounds__(256) pf_prep_kernel(int kvc, int64_t T, int64_t base, int64_t rope_pos0, KvSlot slot,
                                                      const float* __restrict__ q_norm,
                                                      const float* __restrict__ k_norm,
                                                      const float* __restrict__ rope, const Tin* __restrict__ q_gate,
                                                      const Tin* __restrict__ k_in, const Tin* __restrict__ v_in,
                                                      __nv_bfloat16* __restrict__ qb, __nv_bfloat16* __restrict__ kb,
                                                      __nv_bfloat16* __restrict__ vb, int64_t L, float eps) {
    const int64_t t = blockIdx.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nq = GRP * kvc;
    const int64_t pos = base + t;                                   // cache slot
    const float* cs = rope + (rope_pos0 + t) * (2 * ROPE);           // RoPE row of start_pos + t (forward.rs:550-557)
    for (int task = warp; task < nq + kvc; task += 8) {
        const Tin* src;
        const float* w;
        if (task < nq) {
            src = q_gate + (t * nq + task) * QG_ROW;
            w = q_norm;
        } else {
            const int h = task - nq;
            src = k_in + (t * kvc + h) * HD;
            w = k_norm;
            const Tin* vs = v_in + (t * kvc + h) * HD;
            const float4 v0 = ld4<Tin>(vs + 4 * lane), v1 = ld4<Tin>(vs + 128 + 4 * lane);
            float* vd = slot.v + ((size_t)h * slot.cap + pos) * HD;
            reinterpret_cast<float4*>(vd)[lane] = v0;
            reinterpret_cast<float4*>(vd + 128)[lane] = v1;
            __nv_bfloat16* vbd = vb + ((size_t)h * L + pos) * HD;
            st4_bf16(vbd + 4 * lane, v0);
            st4_bf16(vbd + 128 + 4 * lane, v1);
        }
        float4 x0 = ld4<Tin>(src + 4 * lane);
        float4 x1 = ld4<Tin>(src + 128 + 4 * lane);
        float ss = x0.x * x0.x + x0.y * x0.y + x0.z * x0.z + x0.w * x0.w + x1.x * x1.x + x1.y * x1.y +
                   x1.z * x1.z + x1.w * x1.w;
        ss = warp_sum(ss);
        const float inv = 1.0f / sqrtf(ss / (float)HD + eps);
        const float4 w0 = reinterpret_cast<const float4*>(w)[lane];
        const float4 w1 = reinterpret_cast<const float4*>(w)[lane + 32];
        x0 = make_float4((x0.x * inv) * w0.x, (x0.y * inv) * w0.y, (x0.z * inv) * w0.z, (x0.w * inv) * w0.w);
        x1 = make_float4((x1.x * inv) * w1.x, (x1.y * inv) * w1.y, (x1.z * inv) * w1.z, (x1.w * inv) * w1.w);
        float4 pr;
        pr.x = __shfl_xor_sync(0xffffffffu, x0.x, 8);
        pr.y = __shfl_xor_sync(0xffffffffu, x0.y, 8);
        pr.z = __shfl_xor_sync(0xffffffffu, x0.z, 8);
        pr.w = __shfl_xor_sync(0xffffffffu, x0.w, 8);
        if (lane < 16) {
            const float4 c = reinterpret_cast<const float4*>(cs)[lane];
            const float4 s = reinterpret_cast<const float4*>(cs + ROPE)[lane];
            x0 = make_float4(fmaf(x0.x, c.x, pr.x * s.x), fmaf(x0.y, c.y, pr.y * s.y), fmaf(x0.z, c.z, pr.z * s.z),
                             fmaf(x0.w, c.w, pr.w * s.w));
        }
        if (task < nq) {
            // 1/sqrt(256) and log2(e): the attention kernel's scores come out in log2 units
            constexpr float QS = 0.0625f * 1.4426950408889634f;
            x0 = make_float4(x0.x * QS, x0.y * QS, x0.z * QS, x0.w * QS);
            x1 = make_float4(x1.x * QS, x1.y * QS, x1.z * QS, x1.w * QS);
            __nv_bfloat16* qd = qb + ((size_t)task * T + t) * HD;
            st4_bf16(qd + 4 * lane, x0);
            st4_bf16(qd + 128 + 4 * lane, x1);
        } else {
            const int h = task - nq;
            float* kd = slot.k + ((size_t)h * slot.cap + pos) * HD;
            reinterpret_cast<float4*>(kd)[lane] = x0;
            reinterpret_cast<float4*>(kd + 128)[lane] = x1;
            __nv_bfloat16* kbd = kb + ((size_t)h * L + pos) * HD;
            st4_bf16(kbd + 4 * lane, x0);
            st4_bf16(kbd + 128 + 4 * lane, x1);
        }
    }
}

// 2. bf16 copies of rows [0, base) of the f32 cache
__global__ void pf_prior_kernel(int kvc, int64_t base, KvSlot slot, __nv_bfloat16* __restrict__ kb,
                                __nv_bfloat16* __restrict__ vb, int64_t L) {
    const int64_t n4 = (int64_t)kvc * base * (HD / 4);
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t e = i * 4;
        const int64_t h = e / (base * HD);
        const int64_t r = e - h * base * HD;     // row * HD + d
        const float4 kx = *reinterpret_cast<const float4*>(slot.k + (size_t)h * slot.cap * HD + r);
        const float4 vx = *reinterpret_cast<const float4*>(slot.v + (size_t)h * slot.cap * HD + r);
        st4_bf16(kb + (size_t)h * L * HD + r, kx);
        st4_bf16(vb + (size_t)h * L * HD + r, vx);
    }
}

// ---------------------------------------------------------------------------
// 3. attention
// ---------------------------------------------------------------------------
template <typename Tg>
__global__ void __launch_bounds__(pf::NTHREADS, 1) pf_attn_kernel(const __grid_constant__ CUtensorMap tm_q,
                                                                   const __grid_constant__ CUtensorMap tm_k,
                                                                   const __grid_constant__ CUtensorMap tm_v,
                                                                   int kvc, int64_t T, int64_t base,
                                                                   const Tg* __restrict__ q_gate,
                                                                   float* __restrict__ out, int* err,
                                                                   int split_idx, int split_cnt) {
    using namespace pf;
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    // dynamic smem is only guaranteed 16-byte aligned: round up to 1 KB
    // offset the shared-memory pointer itself (integer arithmetic on the address
    // would turn every later access into a generic one)
    Smem& sm = *reinterpret_cast<Smem*>(smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u));
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nq = GRP * kvc;
    const int n_qt = (int)((T + BM - 1) / BM);
    // heaviest (latest) query tiles first; with a split, this context owns the
    // tiles qt % split_cnt == split_idx (interleaved: balanced causal work)
    const int last_own = (n_qt - 1) - (((n_qt - 1) % split_cnt) - split_idx + split_cnt) % split_cnt;
    const int qt = last_own - split_cnt * (int)(blockIdx.x / nq);
    const int qh = (int)(blockIdx.x % nq);
    const int kvh = qh / GRP;
    const int64_t q0 = (int64_t)qt * BM;
    const int64_t q_last = std::min<int64_t>(q0 + BM, T) - 1;         // last valid query row (token index)
    const int nblk = (int)((base + q_last) / BN) + 1;                  // key blocks touching the causal range

    if (warp == 0) {
        tmem_alloc(&sm.tmem_base, 512);
    }
    if (tid == 0) {
        mbar_init(&sm.q_full, 1);
        for (int i = 0; i < NK; ++i) {
            mbar_init(&sm.k_full[i], 1);
            mbar_init(&sm.k_empty[i], 1);
        }
        for (int i = 0; i < NV; ++i) {
            mbar_init(&sm.v_full[i], 1);
            mbar_init(&sm.v_empty[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&sm.s_full[i], 1);
            mbar_init(&sm.p_full[i], 2 * BM);
            mbar_init(&sm.pv_done[i], 1);
        }
        fence_mbar_init();
    }
    fence_before_sync();
    __syncthreads();
    fence_after_sync();
    const uint32_t tmem = sm.tmem_base;
    bool ok = true;

    if (warp == 8) {
        // ---------------- TMA producers: lane 0 = Q and K boxes, lane 1 = V slots ----------------
        if (lane == 0) {
            mbar_arrive_expect_tx(&sm.q_full, BM * HD * 2);
            for (int b = 0; b < 4; ++b) tma_load_3d(&sm.q[b][0][0], &tm_q, 64 * b, (int)q0, qh, &sm.q_full);
            for (int idx = 0; idx < 4 * nblk && ok; ++idx) {
                const int slot = idx % NK, j = idx >> 2, b = idx & 3;
                if (idx >= NK && !wait_or_flag(&sm.k_empty[slot], ((idx / NK) - 1) & 1, err, ok)) break;
                mbar_arrive_expect_tx(&sm.k_full[slot], BN * 64 * 2);
                tma_load_3d(&sm.k[slot][0][0], &tm_k, 64 * b, j * BN, kvh, &sm.k_full[slot]);
            }
        } else if (lane == 1) {
            for (int idx = 0; idx < 4 * nblk && ok; ++idx) {
                const int slot = idx % NV, j = idx >> 2, kg = idx & 3;
                if (idx >= NV && !wait_or_flag(&sm.v_empty[slot], ((idx / NV) - 1) & 1, err, ok)) break;
                mbar_arrive_expect_tx(&sm.v_full[slot], 32 * HD * 2);
                for (int d = 0; d < 4; ++d)
                    tma_load_3d(&sm.v[slot][d][0][0], &tm_v, 64 * d, j * BN + 32 * kg, kvh, &sm.v_full[slot]);
            }
        }
    } else if (warp == 9) {
        // ---------------- MMA issuer (one thread) ----------------
        if (lane == 0) {
            constexpr uint32_t ID_QK = idesc_bf16(BM, BN, false);
            constexpr uint32_t ID_PV = idesc_bf16(BM, HD, true);
            const uint32_t q_s = smem_u32(&sm.q[0][0][0]);
            const uint32_t k_s = smem_u32(&sm.k[0][0][0]);
            const uint32_t v_s = smem_u32(&sm.v[0][0][0][0]);
            auto issue_s = [&](int j) {
                const int st = j & 1;
                for (int b = 0; b < 4; ++b) {
                    const int idx = 4 * j + b, slot = idx % NK;
                    if (!wait_or_flag(&sm.k_full[slot], (idx / NK) & 1, err, ok)) return;
                    fence_after_sync();
#pragma unroll
                    for (int s4 = 0; s4 < 4; ++s4) {
                        const uint32_t off_q = (uint32_t)b * (BM * 128) + (uint32_t)s4 * 32;
                        const uint32_t off_k = (uint32_t)slot * (BN * 128) + (uint32_t)s4 * 32;
                        umma_ss(tmem + S_COL(st), sw128_desc(q_s + off_q, 16, 1024),
                                sw128_desc(k_s + off_k, 16, 1024), ID_QK, (b > 0 || s4 > 0) ? 1u : 0u);
                    }
                    umma_commit(&sm.k_empty[slot]);
                }
                umma_commit(&sm.s_full[st]);
            };
            if (wait_or_flag(&sm.q_full, 0, err, ok)) {
                issue_s(0);
                if (nblk > 1) issue_s(1);
                for (int j = 0; j < nblk && ok; ++j) {
                    const int st = j & 1;
                    if (!wait_or_flag(&sm.p_full[st], (j >> 1) & 1, err, ok)) break;
                    for (int kg = 0; kg < 4 && ok; ++kg) {
                        const int idx = 4 * j + kg, slot = idx % NV;
                        if (!wait_or_flag(&sm.v_full[slot], (idx / NV) & 1, err, ok)) break;
                        fence_after_sync();
#pragma unroll
                        for (int s2 = 0; s2 < 2; ++s2) {
                            // B = V[16 keys][256 dims], MN-major: 64-dim boxes 4 KB apart (LBO),
                            // 8-key swizzle atoms 1 KB apart (SBO); A = P columns of those keys
                            umma_ts(tmem + O_COL, tmem + S_COL(st) + 8 * (2 * kg + s2),
                                    sw128_desc(v_s + (uint32_t)slot * (32 * HD * 2) + (uint32_t)s2 * 16 * 128,
                                               32 * 128, 1024),
                                    ID_PV, (j > 0 || kg > 0 || s2 > 0) ? 1u : 0u);
                        }
                        umma_commit(&sm.v_empty[slot]);
                    }
                    umma_commit(&sm.pv_done[st]);
                    if (j + 2 < nblk) issue_s(j + 2);
                }
            }
        }
    } else {
        // ---------------- softmax: 8 warps, thread = (query row, key half) ----------------
        const int r = 32 * (warp & 3) + lane;               // TMEM lane = query row
        const int hf = warp >> 2;                           // keys [64 hf, 64 hf + 64) of a block
        const uint32_t lane_off = (uint32_t)(32 * (warp & 3)) << 16;
        const int64_t qpos = base + q0 + r;                 // absolute position of this query row
        float m_run = -INFINITY, l_run = 0.0f;              // m identical in both halves; l partial per half
        for (int j = 0; j < nblk; ++j) {
            const int st = j & 1;
            if (!wait_or_flag(&sm.s_full[st], (j >> 1) & 1, err, ok)) break;
            fence_after_sync();
            float s[64];
            {
                uint32_t raw[64];
                tmem_ld32_async(tmem + lane_off + S_COL(st) + 64 * hf, raw);
                tmem_ld32_async(tmem + lane_off + S_COL(st) + 64 * hf + 32, raw + 32);
                tmem_wait_ld();
#pragma unroll
                for (int c = 0; c < 64; ++c) s[c] = __uint_as_float(raw[c]);
            }
            // causal mask: keys k0 + c with c > lim are in the future (only blocks on the diagonal)
            const int64_t lim64 = qpos - ((int64_t)j * BN + 64 * hf);
            if (lim64 < 63) {
                const int lim = lim64 < -1 ? -1 : (int)lim64;
#pragma unroll
                for (int c = 0; c < 64; ++c) s[c] = c > lim ? -INFINITY : s[c];
            }
            float mx;
            {
                float a0 = s[0], a1 = s[1], a2 = s[2], a3 = s[3];
#pragma unroll
                for (int c = 4; c < 64; c += 8) {
                    a0 = max3f(a0, s[c], s[c + 1]);
                    a1 = max3f(a1, s[c + 2], s[c + 3]);
                    a2 = max3f(a2, s[c + 4], s[c + 5]);
                    a3 = max3f(a3, s[c + 6], s[c + 7]);
                }
                mx = fmaxf(max3f(a0, a1, a2), a3);
            }
            sm.red_max[st][hf][r] = mx;
            named_bar_sync(1, 256);                          // also: every S read of this block is done
            mx = fmaxf(mx, sm.red_max[st][hf ^ 1][r]);
            const float m_new = fmaxf(m_run, mx);
            if (m_new > m_run + RESCALE_THRESHOLD) {
                // lazy rescale: the running max moved a lot -- scale l and this half-row of O
                const float f = ex2(m_run - m_new);
                l_run *= f;
                if (j > 0) {
                    const int pj = (j - 1) & 1;
                    if (!wait_or_flag(&sm.pv_done[pj], ((j - 1) >> 1) & 1, err, ok)) break;
                    fence_after_sync();
#pragma unroll 1
                    for (int c = 128 * hf; c < 128 * hf + 128; c += 32) {
                        float o[32];
                        uint32_t ob[32];
                        tmem_ld32(tmem + lane_off + O_COL + c, o);
#pragma unroll
                        for (int i = 0; i < 32; ++i) ob[i] = __float_as_uint(o[i] * f);
                        tmem_st32(tmem + lane_off + O_COL + c, ob);
                    }
                }
                m_run = m_new;
            }
            uint32_t pk[32];
            {
                const uint64_t mm = f2(m_run, m_run);
                uint64_t acc0 = f2(0.0f, 0.0f), acc1 = acc0;
#pragma unroll
                for (int c = 0; c < 64; c += 4) {
                    float x0, x1, x2, x3;
                    f2_split(sub_f2(f2(s[c], s[c + 1]), mm), x0, x1);
                    f2_split(sub_f2(f2(s[c + 2], s[c + 3]), mm), x2, x3);
                    const float p0 = ex2(x0), p1 = ex2(x1), p2 = ex2(x2), p3 = ex2(x3);
                    acc0 = add_f2(acc0, f2(p0, p1));
                    acc1 = add_f2(acc1, f2(p2, p3));
                    pk[c / 2] = pack_bf16(p0, p1);
                    pk[c / 2 + 1] = pack_bf16(p2, p3);
                }
                float u0, u1;
                f2_split(add_f2(acc0, acc1), u0, u1);
                l_run += u0 + u1;
            }
            // P of this block goes over the first 64 columns of its own S buffer (the
            // previous reader of these columns, PV(j-2), completed before S(j) did)
            tmem_st32(tmem + lane_off + S_COL(st) + 32 * hf, pk);
            fence_before_sync();
            mbar_arrive(&sm.p_full[st]);
        }
        // epilogue: O / l * sigmoid(gate); this thread covers dims [128 hf, 128 hf + 128)
        sm.red_l[hf][r] = l_run;
        named_bar_sync(1, 256);
        const float l_tot = l_run + sm.red_l[hf ^ 1][r];
        if (ok) {
            const int jl = nblk - 1;
            if (wait_or_flag(&sm.pv_done[jl & 1], (jl >> 1) & 1, err, ok)) {
                fence_after_sync();
                const int64_t t = q0 + r;
                const float inv_l = 1.0f / l_tot;
#pragma unroll 1
                for (int c = 128 * hf; c < 128 * hf + 128; c += 32) {
                    float o[32];
                    tmem_ld32(tmem + lane_off + O_COL + c, o);
                    if (t < T) {
                        const Tg* g = q_gate + (t * nq + qh) * QG_ROW + HD + c;
                        float* dst = out + (t * nq + qh) * HD + c;
#pragma unroll
                        for (int i = 0; i < 32; i += 4) {
                            const float4 gv = ld4<Tg>(g + i);
                            float4 y;
                            y.x = o[i + 0] * inv_l * sigmoidf_acc(gv.x);
                            y.y = o[i + 1] * inv_l * sigmoidf_acc(gv.y);
                            y.z = o[i + 2] * inv_l * sigmoidf_acc(gv.z);
                            y.w = o[i + 3] * inv_l * sigmoidf_acc(gv.w);
                            *reinterpret_cast<float4*>(dst + i) = y;
                        }
                    }
                }
            }
        }
    }
    fence_before_sync();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tmem, 512);
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
namespace {

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    }
    return fn;
}

// bf16 tensor [d2][d1][256] with a (64 x rows x 1) box, 128-byte swizzle
bool make_map(CUtensorMap* m, const void* base, int64_t d1, int64_t d2, int box_rows) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[3] = {(cuuint64_t)HD, (cuuint64_t)d1, (cuuint64_t)d2};
    cuuint64_t strides[2] = {(cuuint64_t)HD * 2, (cuuint64_t)d1 * HD * 2};
    cuuint32_t box[3] = {64, (cuuint32_t)box_rows, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

cudaError_t launch_gqa_prefill(dz_ctx* ctx, int layer, int seq, int64_t T, int64_t rope_pos0, const uint16_t* q_gate,
                               const uint16_t* k, const uint16_t* v, const float* q_gate_f, const float* k_f,
                               const float* v_f, float* out, cudaStream_t st, int* n_launch) {
    const LayerState& Lr = ctx->layers[layer];
    const int kvc = ctx->cfg.kv_head_count, nq = GRP * kvc;
    const int64_t base = Lr.len[seq];
    const int64_t L = base + T;
    const KvSlot slot = Lr.h_kv[seq];
    const size_t qb_elems = (size_t)nq * T * HD, kb_elems = (size_t)kvc * L * HD;
    cudaError_t e = ensure_prefill_scratch(ctx, (qb_elems + 2 * kb_elems) * 2 + 4096);
    if (e != cudaSuccess) return e;
    __nv_bfloat16* qb = static_cast<__nv_bfloat16*>(ctx->pf);
    __nv_bfloat16* kb = qb + qb_elems;
    __nv_bfloat16* vb = kb + kb_elems;
    const bool bf = q_gate != nullptr;
    if (bf)
        pf_prep_kernel<__nv_bfloat16><<<(unsigned)T, 256, 0, st>>>(
            kvc, T, base, rope_pos0, slot, Lr.q_norm, Lr.k_norm, ctx->rope, reinterpret_cast<const __nv_bfloat16*>(q_gate),
            reinterpret_cast<const __nv_bfloat16*>(k), reinterpret_cast<const __nv_bfloat16*>(v), qb, kb, vb, L,
            ctx->cfg.rms_eps);
    else
        pf_prep_kernel<float><<<(unsigned)T, 256, 0, st>>>(kvc, T, base, rope_pos0, slot, Lr.q_norm, Lr.k_norm, ctx->rope,
                                                          q_gate_f, k_f, v_f, qb, kb, vb, L, ctx->cfg.rms_eps);
    *n_launch += 1;
    if (base > 0) {
        pf_prior_kernel<<<ctx->n_sm * 4, 256, 0, st>>>(kvc, base, slot, kb, vb, L);
        *n_launch += 1;
    }
    CUtensorMap mq, mk, mv;
    if (!make_map(&mq, qb, T, nq, pf::BM) || !make_map(&mk, kb, L, kvc, pf::BN) || !make_map(&mv, vb, L, kvc, 32))
        return cudaErrorInvalidValue;
    const int n_qt = (int)((T + pf::BM - 1) / pf::BM);
    const int sc = ctx->cfg.qtile_split_count, si = ctx->cfg.qtile_split_index;
    const int n_own = n_qt > si ? (n_qt - 1 - si) / sc + 1 : 0;
    const size_t smem = sizeof(pf::Smem) + 1024;
    if (bf) {
        cudaFuncSetAttribute(pf_attn_kernel<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (n_own > 0)
            pf_attn_kernel<__nv_bfloat16><<<n_own * nq, pf::NTHREADS, smem, st>>>(
                mq, mk, mv, kvc, T, base, reinterpret_cast<const __nv_bfloat16*>(q_gate), out, ctx->d_err, si, sc);
    } else {
        cudaFuncSetAttribute(pf_attn_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (n_own > 0)
            pf_attn_kernel<float><<<n_own * nq, pf::NTHREADS, smem, st>>>(mq, mk, mv, kvc, T, base, q_gate_f, out,
                                                                         ctx->d_err, si, sc);
    }
    *n_launch += 1;
    return cudaGetLastError();
}

}  // namespace dz
