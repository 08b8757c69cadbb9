// The activation side of the NVFP4 tensor-core format, per 16-element block: the arithmetic of launch_quantize_nvfp4_lm_out
// (kernel_gb10_nvfp4.cu:1366-1430) in IEEE operations.  Shared by the stand-alone packer and by the RMSNorm kernel of the prompt
// pass, which packs its output row on the way out.
#pragma once

#include <cuda_fp4.h>
#include <cuda_fp8.h>

#include "common.cuh"

namespace q35 {

// block maximum -> the UE4M3 scale byte and the reciprocal of the value it decodes to (0 for an all-zero block)
__device__ __forceinline__ uint8_t nvfp4_act_scale(float amax, float& inv) {
    const float scale_f = fmaxf(__fmul_rn(amax, 1.0f / 6.0f), 1.0f / (float)(1 << 28));
    const __nv_fp8_storage_t s8 = __nv_cvt_float_to_fp8(scale_f, __NV_SATFINITE, __NV_E4M3);
    const __half_raw hr = __nv_cvt_fp8_to_halfraw(s8, __NV_E4M3);
    const float dec = __half2float(*reinterpret_cast<const __half*>(&hr));
    inv = (dec > 0.f) ? __fdiv_rn(1.0f, dec) : 0.f;
    return (uint8_t)s8;
}
// 8 bf16 values (4 words) -> 8 E2M1 nibbles (element 0 in the low nibble of byte 0)
__device__ __forceinline__ uint32_t nvfp4_pack8(const uint32_t (&wd)[4], float inv) {
    uint32_t out = 0;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const float2 f2 = make_float2(__fmul_rn(bf_lo(wd[k]), inv), __fmul_rn(bf_hi(wd[k]), inv));
        out |= (uint32_t)(uint8_t)__nv_cvt_float2_to_fp4x2(f2, __NV_E2M1, cudaRoundNearest) << (8 * k);
    }
    return out;
}
__device__ __forceinline__ float nvfp4_amax8(const uint32_t (&wd)[4]) {
    float amax = 0.f;
#pragma unroll
    for (int k = 0; k < 4; ++k) amax = fmaxf(amax, fmaxf(fabsf(bf_lo(wd[k])), fabsf(bf_hi(wd[k]))));
    return amax;
}
// where the scale byte of block `blk` (16 elements) of row `row` lives: 512-byte atoms of 128 rows x 4 blocks, the atoms of
// one 128-row group consecutive along K
__device__ __forceinline__ size_t nvfp4_scale_index(long long row, int blk, int K) {
    return (size_t)((row >> 7) * (K / 64) + (blk >> 2)) * 512 + (size_t)((row & 31) * 16 + ((row & 127) >> 5) * 4 + (blk & 3));
}

}  // namespace q35
