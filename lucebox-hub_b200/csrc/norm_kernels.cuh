// Row norms shared by the 27B-class paths (tree verify, draft forward): block sum and RMSNorm with plain weights.
#pragma once

#include "common.cuh"

namespace q35 {

// ---------------------------------------------- norms ----------------------------------------------
__device__ __forceinline__ float tv_block_sum(float v, float* red) {
    v = warp_sum(v);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float t = 0.f;
    for (int i = 0; i < nw; ++i) t += red[i];
    return t;
}

// y = bf16(x * rsqrt(mean x^2 + eps) * w), w f32 applied as a plain multiply (qwen35_target_graph.cpp:260-264)
static __global__ void __launch_bounds__(256) tv_rmsnorm_kernel(const bf16* __restrict__ x, const float* __restrict__ w, bf16* __restrict__ out, int H, float eps) {
    // H is a multiple of 256; a thread keeps its (up to 4) 8-element pieces of the row in registers between the two passes
    __shared__ float red[8];
    constexpr int MAXV = 4;
    pdl_trigger();      // the projection GEMM that follows loads and dequantises its first weights beside this kernel
    pdl_wait();
    const uint4* xr = reinterpret_cast<const uint4*>(x + (size_t)blockIdx.x * H);
    const int nv = H / 8;
    uint4 v[MAXV];
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < MAXV; ++j) {
        const int i = threadIdx.x + j * 256;
        if (i < nv) {
            v[j] = xr[i];
            const bf16* e = reinterpret_cast<const bf16*>(&v[j]);
#pragma unroll
            for (int k = 0; k < 8; ++k) { const float f = bf2f(e[k]); ss = fmaf(f, f, ss); }
        }
    }
    for (int i = threadIdx.x + MAXV * 256; i < nv; i += 256) {          // rows wider than 8192: the tail is read twice
        const uint4 t = xr[i];
        const bf16* e = reinterpret_cast<const bf16*>(&t);
#pragma unroll
        for (int k = 0; k < 8; ++k) { const float f = bf2f(e[k]); ss = fmaf(f, f, ss); }
    }
    const float inv = rsqrt_ieee(tv_block_sum(ss, red) / (float)H + eps);
    uint4* orow = reinterpret_cast<uint4*>(out + (size_t)blockIdx.x * H);
    auto emit = [&](int i, const uint4& t) {
        const bf16* e = reinterpret_cast<const bf16*>(&t);
        const float4 w0 = *reinterpret_cast<const float4*>(w + (size_t)i * 8), w1 = *reinterpret_cast<const float4*>(w + (size_t)i * 8 + 4);
        const float ws[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
        uint4 o;
        bf16* oe = reinterpret_cast<bf16*>(&o);
#pragma unroll
        for (int k = 0; k < 8; ++k) oe[k] = f2bf(bf2f(e[k]) * inv * ws[k]);
        orow[i] = o;
    };
#pragma unroll
    for (int j = 0; j < MAXV; ++j) {
        const int i = threadIdx.x + j * 256;
        if (i < nv) emit(i, v[j]);
    }
    for (int i = threadIdx.x + MAXV * 256; i < nv; i += 256) emit(i, xr[i]);
}

}  // namespace q35
