// dz_common.cuh -- shared constants and sm_100a PTX helpers for libdzattn.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace dz {

// Bonsai-27B shapes (Daiza-engine/src/model/config.rs:47-74)
constexpr int HQ = 24, HKV = 4, GRP = 6, HD = 256, ROPE = 64;
constexpr int SSM_HK = 16, SSM_HV = 48, SSM_D = 128, CONV_K = 4;
constexpr int QKD = SSM_HK * SSM_D;         // 2048
constexpr int INNER = SSM_HV * SSM_D;       // 6144
constexpr int QKV_LEN = 2 * QKD + INNER;    // 10240
constexpr int QG_ROW = 2 * HD;              // one [Q_h | gate_h] head row (512)

constexpr float LOG2E = 1.4426950408889634f;

// Device-side error word: kernels that give up on a bounded wait record a
// code here and return instead of hanging (read by dz_device_error()).
enum : int { DEVERR_NONE = 0, DEVERR_MBAR_TIMEOUT = 1 };

// Time limit for an mbarrier wait, read from the %globaltimer nanosecond clock.
// Every legitimate wait in these kernels (a bulk copy, a tensor-core product,
// another warp's epilogue) ends within microseconds; one second means the
// phase will never complete.
constexpr uint64_t MBAR_WAIT_LIMIT_NS = 1000000000ull;

__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;"
                 ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

// try_wait suspends the thread in hardware until the phase completes or the
// hint (ns) runs out, so waiting warps do not spin on the issue slots that the
// working warps of the same sub-partition need.
constexpr uint32_t MBAR_SUSPEND_HINT_NS = 100000;

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity), "r"(MBAR_SUSPEND_HINT_NS) : "memory");
    return ok != 0;
}

// Bounded wait.  Returns false (and records DEVERR_MBAR_TIMEOUT) if the phase
// did not complete within MBAR_WAIT_LIMIT_NS.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_ns();
    for (uint32_t i = 1;; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 15u) == 0 && global_ns() - t0 > MBAR_WAIT_LIMIT_NS) break;
    }
    if (err) atomicExch(err, DEVERR_MBAR_TIMEOUT);
    return false;
}

// 1-D bulk async copy global -> shared, completion counted on an mbarrier.
// Both addresses 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst_smem, const void* src_gmem, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
        ::"r"(smem_u32(dst_smem)), "l"(src_gmem), "r"(bytes), "r"(smem_u32(bar)) : "memory");
}

// 1-D bulk async copy shared -> global (bulk-group completion).
__device__ __forceinline__ void bulk_s2g(void* dst_gmem, const void* src_smem, uint32_t bytes) {
    asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;"
                 ::"l"(dst_gmem), "r"(smem_u32(src_smem)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
// Make generic-proxy shared-memory writes visible to the async (bulk/TMA) proxy.
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

__device__ __forceinline__ float sigmoidf_acc(float x) { return 1.0f / (1.0f + expf(-x)); }
__device__ __forceinline__ float siluf_acc(float x) { return x / (1.0f + expf(-x)); }
// softplus as the reference defines it (model/ssm.rs:61-67)
__device__ __forceinline__ float softplus_ref(float x) { return x > 20.0f ? x : logf(1.0f + expf(x)); }

}  // namespace dz
