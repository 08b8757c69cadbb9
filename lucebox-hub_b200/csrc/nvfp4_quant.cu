// NVFP4 weight packers (E2M1 values with block scales), both layouts of the reference:
//   * decode-body layout   quantize_nvfp4_kernel,    kernel_gb10_nvfp4.cu:1742-1810, launcher :1863-1876
//     groups of `group_size` (default 32) along K, fp16 scale = amax/6 (1.0 for an all-zero group), fixed
//     thresholds with ties going up, low nibble = even element, scales row-major [rows, cols/group_size];
//   * tensor-core layout   quantize_nvfp4_lm_kernel, kernel_gb10_nvfp4.cu:1366-1430, launcher :1878-1892
//     16-element blocks, UE4M3 scale = sat_rn(max(amax/6, 2^-28)), elements divided by the decoded scale and
//     rounded to E2M1 with round-to-nearest-even, scale bytes in 128-row x 4-column tiles of 512 bytes.
// Pure streaming kernels: one 16-byte (or 2 x 16-byte) load per thread, coalesced along K.
// The packed bytes must equal those of the reference's own kernels, and the reference builds with --use_fast_math
// (models/qwen35_0p8b/setup.py): its `amax / 6.0f`, `1.0f / scale` and `1.0f / decoded_scale` are approximate divisions
// and reciprocals.  This file is therefore compiled with --use_fast_math too (build.py) and writes those three
// expressions in the reference's form, so the compiler lowers them the same way; everything else in it is exact
// either way (comparisons, products of two floats, conversions).  tests/test_nvfp4_gpu.py compares the bytes with the
// reference's kernels compiled from its own source; the IEEE restatement in oracle/nvfp4_ref.py differs from both in the
// rare element that sits on a rounding boundary of the approximate reciprocal.
#include <cuda_fp16.h>
#include <cuda_fp4.h>
#include <cuda_fp8.h>

#include "common.cuh"
#include "runtime.h"

namespace q35 {

__device__ __forceinline__ unsigned fp4_threshold_code(float x) {
    const float ax = fabsf(x);
    unsigned mag = ax < 0.25f ? 0u : ax < 0.75f ? 1u : ax < 1.25f ? 2u : ax < 1.75f ? 3u : ax < 2.5f ? 4u : ax < 3.5f ? 5u : ax < 5.0f ? 6u : 7u;
    return (x < 0.0f) ? (mag | 8u) : mag;
}

// one thread per group of `group_size` elements (a multiple of 8)
__global__ void __launch_bounds__(256) quantize_nvfp4_kernel(const bf16* __restrict__ w, uint8_t* __restrict__ packed,
                                                             __half* __restrict__ scales, long long total_groups, int cols, int group_size) {
    const int gpr = cols / group_size;
    for (long long gid = (long long)blockIdx.x * blockDim.x + threadIdx.x; gid < total_groups; gid += (long long)gridDim.x * blockDim.x) {
        const long long row = gid / gpr;
        const int grp = (int)(gid % gpr);
        const uint4* src = reinterpret_cast<const uint4*>(w + row * cols + (long long)grp * group_size);
        uint8_t* dst = packed + row * (cols / 2) + grp * (group_size / 2);
        float amax = 0.f;
        for (int i = 0; i < group_size / 8; ++i) {
            const uint4 v = __ldg(src + i);
            amax = fmaxf(amax, fmaxf(fmaxf(fabsf(bf_lo(v.x)), fabsf(bf_hi(v.x))), fmaxf(fabsf(bf_lo(v.y)), fabsf(bf_hi(v.y)))));
            amax = fmaxf(amax, fmaxf(fmaxf(fabsf(bf_lo(v.z)), fabsf(bf_hi(v.z))), fmaxf(fabsf(bf_lo(v.w)), fabsf(bf_hi(v.w)))));
        }
        const float scale = (amax > 0.0f) ? (amax / 6.0f) : 1.0f;          // kernel_gb10_nvfp4.cu:1791
        scales[gid] = __float2half(scale);
        const float inv = 1.0f / scale;                                    // :1801
        for (int i = 0; i < group_size / 8; ++i) {
            const uint4 v = __ldg(src + i);
            const uint32_t wd[4] = {v.x, v.y, v.z, v.w};
            uint32_t out = 0;
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const unsigned lo = (amax > 0.f) ? fp4_threshold_code(bf_lo(wd[k]) * inv) : 0u;
                const unsigned hi = (amax > 0.f) ? fp4_threshold_code(bf_hi(wd[k]) * inv) : 0u;
                out |= (lo | (hi << 4)) << (8 * k);
            }
            reinterpret_cast<uint32_t*>(dst)[i] = out;
        }
    }
}

// one thread per 16-element block
__global__ void __launch_bounds__(256) quantize_nvfp4_lm_kernel(const bf16* __restrict__ w, uint8_t* __restrict__ packed,
                                                                uint8_t* __restrict__ scales, long long total_blocks, int cols) {
    const int bpr = cols / 16;
    for (long long bid = (long long)blockIdx.x * blockDim.x + threadIdx.x; bid < total_blocks; bid += (long long)gridDim.x * blockDim.x) {
        const long long row = bid / bpr;
        const int sc = (int)(bid % bpr);
        const uint4* src = reinterpret_cast<const uint4*>(w + row * cols + sc * 16);
        const uint4 v0 = __ldg(src), v1 = __ldg(src + 1);
        const uint32_t wd[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
        float amax = 0.f;
#pragma unroll
        for (int k = 0; k < 8; ++k) amax = fmaxf(amax, fmaxf(fabsf(bf_lo(wd[k])), fabsf(bf_hi(wd[k]))));
        const float scale_f = fmaxf(amax * (1.0f / 6.0f), 1.0f / float(1 << 28));   // kernel_gb10_nvfp4.cu:1402
        const __nv_fp8_storage_t s8 = __nv_cvt_float_to_fp8(scale_f, __NV_SATFINITE, __NV_E4M3);
        const __half_raw hr = __nv_cvt_fp8_to_halfraw(s8, __NV_E4M3);
        const float dec = __half2float(*reinterpret_cast<const __half*>(&hr));
        const float inv = (dec > 0.0f) ? (1.0f / dec) : 0.0f;                       // :1406
        unsigned long long out = 0;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const float2 f2 = make_float2(bf_lo(wd[k]) * inv, bf_hi(wd[k]) * inv);
            const __nv_fp4x2_storage_t p = __nv_cvt_float2_to_fp4x2(f2, __NV_E2M1, cudaRoundNearest);
            out |= (unsigned long long)(uint8_t)p << (8 * k);
        }
        *reinterpret_cast<unsigned long long*>(packed + row * (cols / 2) + sc * 8) = out;
        const long long tile = (row >> 7) * (cols / 64) + (sc >> 2);
        scales[tile * 512 + (row & 31) * 16 + ((row & 127) >> 5) * 4 + (sc & 3)] = (uint8_t)s8;
    }
}

}  // namespace q35

extern "C" int launch_quantize_nvfp4_out(const void* weight, int rows, int cols, int group_size, void* packed_out, void* scales_out,
                                         qwen35_stream_t stream) {
    using namespace q35;
    if (!weight || !packed_out || !scales_out || rows <= 0 || cols <= 0 || group_size <= 0 || group_size % 8 != 0 || cols % group_size != 0) {
        set_error("quantize_nvfp4: cols (%d) must be a multiple of group_size (%d), group_size a multiple of 8", cols, group_size);
        return QWEN35_ERR_BAD_ARG;
    }
    const long long groups = (long long)rows * (cols / group_size);
    const int blocks = (int)((groups + 255) / 256 < 148 * 16 ? (groups + 255) / 256 : 148 * 16);
    quantize_nvfp4_kernel<<<blocks, 256, 0, (cudaStream_t)stream>>>((const bf16*)weight, (uint8_t*)packed_out, (__half*)scales_out, groups, cols, group_size);
    Q35_CUDA_OK(cudaGetLastError());
    g_launches.fetch_add(1);
    return QWEN35_OK;
}

extern "C" int launch_quantize_nvfp4_lm_out(const void* weight, int rows, int cols, void* packed_out, void* scales_out, qwen35_stream_t stream) {
    using namespace q35;
    if (!weight || !packed_out || !scales_out || rows <= 0 || rows % 128 != 0 || cols <= 0 || cols % 64 != 0) {
        set_error("quantize_nvfp4_lm: rows (%d) must be a multiple of 128 and cols (%d) a multiple of 64", rows, cols);
        return QWEN35_ERR_BAD_ARG;
    }
    const long long nblk = (long long)rows * (cols / 16);
    const int blocks = (int)((nblk + 255) / 256 < 148 * 16 ? (nblk + 255) / 256 : 148 * 16);
    quantize_nvfp4_lm_kernel<<<blocks, 256, 0, (cudaStream_t)stream>>>((const bf16*)weight, (uint8_t*)packed_out, (uint8_t*)scales_out, nblk, cols);
    Q35_CUDA_OK(cudaGetLastError());
    g_launches.fetch_add(1);
    return QWEN35_OK;
}
