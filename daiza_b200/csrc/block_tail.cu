// block_tail.cu -- the elementwise steps of a block's tail around the Q1_0
// GEMVs (dz_block_mlp in dz_attn.cu strings them together).
//
// Reference: Daiza-engine/src/model/block.rs:93-104 (post_attention_norm =
// math/rmsnorm.rs:180-202 rmsnorm_into: (x * inv_rms) * w with
// inv_rms = 1 / sqrt(sum x^2 / n + eps)), mlp.rs:48 (swiglu_inplace,
// math/simd_exp.rs:273-296: gate = silu(gate) * up).
#include "dz_internal.h"

namespace dz {

// one CTA of 256 threads per row
__global__ void __launch_bounds__(256) rmsnorm_rows_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                                           float eps, int n, float* __restrict__ out) {
    __shared__ float red[8];
    asm volatile("griddepcontrol.launch_dependents;");
    const int row = blockIdx.x, tid = threadIdx.x;
    const float4* xr = reinterpret_cast<const float4*>(x + (size_t)row * n);
    float ss = 0.0f;
    for (int i = tid; i < n / 4; i += 256) {
        const float4 v = xr[i];
        ss = fmaf(v.x, v.x, fmaf(v.y, v.y, fmaf(v.z, v.z, fmaf(v.w, v.w, ss))));
    }
    ss = warp_sum(ss);
    if ((tid & 31) == 0) red[tid >> 5] = ss;
    __syncthreads();
    float tot = 0.0f;
#pragma unroll
    for (int k = 0; k < 8; ++k) tot += red[k];
    const float inv = 1.0f / sqrtf(tot / (float)n + eps);
    const float4* wr = reinterpret_cast<const float4*>(w);
    float4* o = reinterpret_cast<float4*>(out + (size_t)row * n);
    for (int i = tid; i < n / 4; i += 256) {
        const float4 v = xr[i], ww = wr[i];
        o[i] = make_float4((v.x * inv) * ww.x, (v.y * inv) * ww.y, (v.z * inv) * ww.z, (v.w * inv) * ww.w);
    }
}

__global__ void swiglu_kernel(float* __restrict__ gate, const float* __restrict__ up, int64_t n4) {
    asm volatile("griddepcontrol.launch_dependents;");
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
        float4 g = reinterpret_cast<float4*>(gate)[i];
        const float4 u = reinterpret_cast<const float4*>(up)[i];
        g = make_float4(siluf_acc(g.x) * u.x, siluf_acc(g.y) * u.y, siluf_acc(g.z) * u.z, siluf_acc(g.w) * u.w);
        reinterpret_cast<float4*>(gate)[i] = g;
    }
}

cudaError_t launch_rmsnorm_rows(const float* x, const float* w, float eps, int T, int n, float* out, cudaStream_t st) {
    rmsnorm_rows_kernel<<<T, 256, 0, st>>>(x, w, eps, n, out);
    return cudaGetLastError();
}

cudaError_t launch_swiglu(float* gate, const float* up, int64_t n, cudaStream_t st) {
    const int64_t n4 = n / 4;
    const int grid = (int)std::min<int64_t>((n4 + 255) / 256, 148 * 8);
    swiglu_kernel<<<grid, 256, 0, st>>>(gate, up, n4);
    return cudaGetLastError();
}

}  // namespace dz
