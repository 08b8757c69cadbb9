// Known-answer generator for the NVFP4 packers' number formats.  TEST INFRASTRUCTURE ONLY.
// Calls the host implementations of NVIDIA's conversion functions -- the same functions the
// reference packer calls on the device (kernel_gb10_nvfp4.cu:1398-1412) -- and prints, for a list of
// floats read from stdin (one hex bit pattern per line), the E4M3 byte, its decoded value and the E2M1 code.
// Build: see oracle/Makefile (g++ with the CUDA include directory; no GPU needed).
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cuda_fp4.h>

#include <cstdint>
#include <cstdio>
#include <cstring>

int main() {
    unsigned int bits;
    while (scanf("%x", &bits) == 1) {
        float f;
        memcpy(&f, &bits, 4);
        const __nv_fp8_storage_t e4 = __nv_cvt_float_to_fp8(f, __NV_SATFINITE, __NV_E4M3);
        const __half_raw hr = __nv_cvt_fp8_to_halfraw(e4, __NV_E4M3);
        __half h;
        memcpy(&h, &hr, 2);
        const float dec = __half2float(h);
        unsigned int dbits;
        memcpy(&dbits, &dec, 4);
        float2 v;
        v.x = f;
        v.y = 0.0f;
        const __nv_fp4x2_storage_t p = __nv_cvt_float2_to_fp4x2(v, __NV_E2M1, cudaRoundNearest);
        printf("%08x %02x %08x %x\n", bits, (unsigned)e4, dbits, (unsigned)p & 0xfu);
    }
    return 0;
}
