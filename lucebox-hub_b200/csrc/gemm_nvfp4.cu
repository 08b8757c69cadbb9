// NVFP4 block-scaled GEMM on the 5th-generation tensor cores:  C[T, N] = alpha * (A_q . W_q^T), both operands E2M1 with one
// UE4M3 scale per 16 elements along K, f32 accumulation in tensor memory (tcgen05.mma kind::mxf4nvf4, block16).
//
// Replaces the reference's cuBLASLt NVFP4 calls: the FP4 LM head (launch_lm_head_from_f32_normalized and its plan,
// kernel_gb10_nvfp4.cu:277-473, 1894-1997: hidden padded to 16 rows, activation quantised to FP4 as well) and the NVFP4
// prefill projections (cublaslt_nvfp4_bf16_gemm, prefill.cu:1020-1155).  Operand formats are the reference's "tensor-core"
// pack (launch_quantize_nvfp4_lm_out): packed nibbles [rows, K/2], low nibble = even element, and scale bytes in 512-byte
// atoms of 128 rows x 4 scales (byte = (row % 32) * 16 + (row % 128 / 32) * 4 + scale % 4), atoms of one 128-row block
// consecutive along K.  That atom IS the shared-memory image tcgen05.cp (32x128b, warpx4) moves into tensor memory as the
// scale-factor operand of one K = 64 instruction, so weights packed for the reference run here without repacking.
//
// The weight matrix is the M operand (128 rows of W per CTA fill the 128 accumulator lanes); the tokens are the N operand
// (T_TILE = 16 ... 128 per CTA), so a 16-row LM-head problem wastes nothing.  Per CTA:
//   warp 0   producer: per 256-wide k-step one 128B-swizzled TMA box of packed weights (128 rows x 128 bytes), one of packed
//            activations (T_TILE rows x 128 bytes) and two 2 KB bulk copies of scale atoms (4 K-atoms each)
//   warp 1   allocates tensor memory; one thread copies the 8 scale atoms of the stage into tensor memory and issues the
//            four K = 64 instructions, then commits the stage back to the producer
//   warps 2-5 epilogue: tcgen05.ld rows of the accumulator (lane = weight row, column = token), scale, round once to bf16
//            and park the tile transposed, [token][weight row], in the idle stage buffers; then all six warps store whole
//            rows of C (16 bytes per thread, residual added there).  f32 output (the 16-row LM head) is stored directly.
// Every wait is bounded; a wait that runs out sets the status word and the CTA unwinds normally.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_fp16.h>
#include <cuda_fp4.h>
#include <cuda_fp8.h>

#include "common.cuh"
#include "nvfp4_act.cuh"
#include "runtime.h"

namespace q35 {

constexpr int FP4_BM = 128;                     // weight rows per CTA
constexpr int FP4_BK = 256;                     // elements of K per stage = 128 bytes of packed nibbles per row
// stages per CTA: three of 36 KB for the 128-token tile, so that two CTAs share an SM (the epilogue of one tile runs under the
// main loop of another; 256 tensor-memory columns each), four for the narrower tiles
__host__ __device__ constexpr int fp4_stages(int t_tile) { return t_tile >= 128 ? 3 : 4; }
// bf16 results are parked [token][FP4_PARK_LD] in the idle stage buffers and stored as whole rows
constexpr int FP4_PARK_LD = FP4_BM + 8;
constexpr int FP4_THREADS = 192;
constexpr uint32_t FP4_W_BYTES = FP4_BM * 128;  // 16 KB
constexpr uint32_t FP4_SF_BYTES = 4 * 512;      // four K-atoms of scales per stage and operand
constexpr unsigned FP4_SPIN_LIMIT = 20u * 1000u * 1000u;
constexpr uint32_t FP4_TMEM_COLS = 256;         // accumulator (<= 128) + two alternating sets of 32 scale columns

__host__ __device__ constexpr uint32_t fp4_stage_bytes(int t_tile) { return FP4_W_BYTES + (uint32_t)t_tile * 128u + 2u * FP4_SF_BYTES; }
__host__ __device__ constexpr uint32_t fp4_park_bytes(int t_tile) { return (uint32_t)t_tile * FP4_PARK_LD * 2u; }
__host__ __device__ constexpr uint32_t fp4_tile_bytes(int t_tile) {
    return fp4_stages(t_tile) * fp4_stage_bytes(t_tile) > fp4_park_bytes(t_tile) ? fp4_stages(t_tile) * fp4_stage_bytes(t_tile)
                                                                                  : ((fp4_park_bytes(t_tile) + 1023u) & ~1023u);
}
__host__ __device__ constexpr uint32_t fp4_smem(int t_tile) { return fp4_tile_bytes(t_tile) + 1024 + 256; }

struct Fp4GemmParams {
    int T, N, K;                 // tokens, output columns (<= the weight rows the tensor map covers), reduction length
    void* C; int ldc;            // [T][ldc], bf16 (out_f32 = 0) or f32 (out_f32 = 1)
    const bf16* R; int ldr;      // optional residual, bf16 [T][ldr] (added after the rounding to bf16)
    const uint8_t* w_scales;     // atoms [N/128][K/64][512]
    const uint8_t* a_scales;     // atoms [ceil(T/128)][K/64][512]
    float alpha;                 // per-tensor scale product
    int out_f32;
    int* err;
};

__device__ __forceinline__ uint32_t f_smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ bool f_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile("{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
                 : "=r"(ok) : "r"(bar), "r"(parity) : "memory");
    return ok != 0;
}
__device__ __forceinline__ bool f_wait(uint32_t bar, uint32_t parity, int* err, volatile int* s_abort) {
    unsigned it = 0;
    while (!f_try_wait(bar, parity)) {
        if (*s_abort) return false;
        if (++it > FP4_SPIN_LIMIT) { *s_abort = 1; atomicCAS(err, 0, (int)ERR_BARRIER_TIMEOUT); return false; }
    }
    return true;
}
// K-major operand tile, 128-byte swizzle: start address >> 4 | SBO = 1024 B between 8-row groups | version 1 | layout 2
__device__ __forceinline__ uint64_t f_desc_sw128(uint32_t smem_addr) {
    return (uint64_t)((smem_addr & 0x3FFFFu) >> 4) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) | ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
// one scale atom: 32 rows of 16 bytes, no swizzle: 8-row core matrices 128 bytes apart
__device__ __forceinline__ uint64_t f_desc_sf_atom(uint32_t smem_addr) {
    return (uint64_t)((smem_addr & 0x3FFFFu) >> 4) | ((uint64_t)(128 >> 4) << 32) | ((uint64_t)1 << 46);
}
// instruction descriptor of the block-scaled MMA: A and B E2M1 (format 1) K-major, scales UE4M3 (bit 23 = 0), N >> 3 at [17,23),
// M >> 4 at [24,29), K = 64 (bit 31 = 0); the scale-factor ids ([4,6) and [29,31)) are the byte offsets inside a 32-bit
// tensor-memory column and are zero for block16 (all four bytes of the column are used)
__device__ __forceinline__ uint32_t f_idesc(int n) {
    return (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(FP4_BM >> 4) << 24);
}

template <int T_TILE>
__global__ void __launch_bounds__(FP4_THREADS, 2)
gemm_nvfp4_tcgen05_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmA, const Fp4GemmParams p) {
    static_assert(T_TILE % 16 == 0 && T_TILE >= 16 && T_TILE <= 128, "token tile: a multiple of 16 up to 128");
    constexpr uint32_t STAGE = fp4_stage_bytes(T_TILE);
    constexpr int FP4_STAGES = fp4_stages(T_TILE);
    constexpr uint32_t A_OFF = FP4_W_BYTES, SFW_OFF = A_OFF + T_TILE * 128u, SFA_OFF = SFW_OFF + FP4_SF_BYTES;
    extern __shared__ unsigned char f_smem_raw[];
    const uint32_t raw = f_smem_u32(f_smem_raw);
    const uint32_t tiles = (raw + 1023u) & ~1023u;                 // swizzled tiles need 1024-byte alignment
    unsigned char* tiles_ptr = f_smem_raw + (tiles - raw);
    uint64_t* bars = reinterpret_cast<uint64_t*>(tiles_ptr + fp4_tile_bytes(T_TILE));
    const uint32_t full0 = f_smem_u32(bars), empty0 = full0 + 8 * FP4_STAGES, tfull = empty0 + 8 * FP4_STAGES;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * FP4_STAGES + 1);
    volatile int* s_abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n0 = blockIdx.x * FP4_BM, t0 = blockIdx.y * T_TILE;
    const int nkb = p.K / FP4_BK;

    if (threadIdx.x == 0) {
        asm volatile("prefetch.tensormap [%0];" ::"l"(&tmW) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(&tmA) : "memory");
        *s_abort = 0;
        for (int i = 0; i < FP4_STAGES; ++i) {
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(full0 + 8 * i) : "memory");
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(empty0 + 8 * i) : "memory");
        }
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(tfull) : "memory");
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(f_smem_u32(tmem_slot)), "r"(FP4_TMEM_COLS) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem_base = *tmem_slot;
    pdl_wait();

    if (warp == 0) {
        if (lane == 0) {
            int issued = 0;
            const uint8_t* sfw = p.w_scales + (size_t)blockIdx.x * (p.K / 64) * 512;
            const uint8_t* sfa = p.a_scales + (size_t)(t0 / 128) * (p.K / 64) * 512;
            for (int i = 0; i < nkb; ++i) {
                const int st = i % FP4_STAGES;
                if (!f_wait(empty0 + 8 * st, ((i / FP4_STAGES) & 1) ^ 1, p.err, s_abort)) break;
                const uint32_t dst = tiles + st * STAGE, bar = full0 + 8 * st;
                asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(STAGE) : "memory");
                asm volatile("cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
                             ::"r"(dst), "l"(&tmW), "r"(i * 128), "r"(n0), "r"(bar) : "memory");
                asm volatile("cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
                             ::"r"(dst + A_OFF), "l"(&tmA), "r"(i * 128), "r"(t0), "r"(bar) : "memory");
                asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                             ::"r"(dst + SFW_OFF), "l"(sfw + (size_t)i * FP4_SF_BYTES), "r"(FP4_SF_BYTES), "r"(bar) : "memory");
                asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                             ::"r"(dst + SFA_OFF), "l"(sfa + (size_t)i * FP4_SF_BYTES), "r"(FP4_SF_BYTES), "r"(bar) : "memory");
                issued = i + 1;
            }
            if (*s_abort) {      // every copy this CTA issued must have landed before it may exit
                for (int i = max(0, issued - FP4_STAGES); i < issued; ++i) {
                    unsigned it = 0;
                    while (!f_try_wait(full0 + 8 * (i % FP4_STAGES), (i / FP4_STAGES) & 1) && ++it < FP4_SPIN_LIMIT) {}
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            const uint32_t idesc = f_idesc(T_TILE);
            for (int i = 0; i < nkb; ++i) {
                const int st = i % FP4_STAGES;
                if (!f_wait(full0 + 8 * st, (i / FP4_STAGES) & 1, p.err, s_abort)) break;
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const uint32_t w_addr = tiles + st * STAGE;
                // scale columns: set (i & 1): weights at [128 + 32 set, +16), activations at [+16, +32); atom k takes 4 columns
                const uint32_t sf_col = tmem_base + 128u + 32u * (uint32_t)(i & 1);
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(sf_col + 4u * k), "l"(f_desc_sf_atom(w_addr + SFW_OFF + 512u * k)) : "memory");
                    asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(sf_col + 16u + 4u * k), "l"(f_desc_sf_atom(w_addr + SFA_OFF + 512u * k)) : "memory");
                }
                const uint64_t wdesc = f_desc_sw128(w_addr), adesc = f_desc_sw128(w_addr + A_OFF);
#pragma unroll
                for (int k = 0; k < 4; ++k) {        // 64 elements = 32 bytes of K per instruction: the start-address field advances by 2
                    const uint32_t acc = (i > 0 || k > 0) ? 1u : 0u;
                    asm volatile(
                        "{\n\t.reg .pred p;\n\t"
                        "setp.ne.b32 p, %4, 0;\n\t"
                        "tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.block16 [%0], %1, %2, %3, [%5], [%6], p;\n\t}"
                        ::"r"(tmem_base), "l"(wdesc + (uint64_t)(2 * k)), "l"(adesc + (uint64_t)(2 * k)), "r"(idesc), "r"(acc),
                          "r"(sf_col + 4u * k), "r"(sf_col + 16u + 4u * k) : "memory");
                }
                asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(empty0 + 8 * st) : "memory");
            }
            asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(tfull) : "memory");
        }
    } else {
        // ---- epilogue: warp w may touch tensor-memory lanes [32 (w % 4), +32): lane = weight row, column = token ----
        const int q = warp & 3;
        const int col = n0 + q * 32 + lane;                        // output column (weight row)
        const bool ok = __all_sync(0xffffffffu, f_wait(tfull, 0, p.err, s_abort) && !*s_abort);
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        if (ok) {
            bf16* park = reinterpret_cast<bf16*>(tiles_ptr);
#pragma unroll
            for (int c = 0; c < T_TILE / 16; ++c) {
                uint32_t v[16];
                asm volatile(
                    "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
                    : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
                      "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
                    : "r"(tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(c * 16)) : "memory");
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
                if (p.out_f32) {
                    if (col < p.N) {
#pragma unroll
                        for (int j = 0; j < 16; ++j) {
                            const int tok = t0 + c * 16 + j;
                            if (tok < p.T) reinterpret_cast<float*>(p.C)[(size_t)tok * p.ldc + col] = __uint_as_float(v[j]) * p.alpha;
                        }
                    }
                } else {
                    // the 32 lanes of a warp write 32 adjacent bf16 of one token's row: conflict-free
#pragma unroll
                    for (int j = 0; j < 16; ++j) park[(c * 16 + j) * FP4_PARK_LD + q * 32 + lane] = f2bf(__uint_as_float(v[j]) * p.alpha);
                }
            }
        }
    }
    __syncthreads();                                              // the parked tile is complete (all warps pass here, whatever happened)
    if (!p.out_f32 && !*s_abort) {
        // ---- store pass, all six warps: a work item is one token x 8 adjacent output columns (16 bytes) ----
        const bf16* park = reinterpret_cast<const bf16*>(tiles_ptr);
        constexpr int NG = FP4_BM / 8;
        const int t = (int)threadIdx.x, cg = (t % NG) * 8, r_first = t / NG, r_step = FP4_THREADS / NG;
        const int rows = min(T_TILE, p.T - t0);
        bf16* cbase = reinterpret_cast<bf16*>(p.C);
        const bool vec_ok = n0 + cg + 8 <= p.N && ((reinterpret_cast<uintptr_t>(cbase + n0 + cg) | (size_t)p.ldc * 2) & 15) == 0 &&
                            (!p.R || ((reinterpret_cast<uintptr_t>(p.R + n0 + cg) | (size_t)p.ldr * 2) & 15) == 0);
        for (int r = r_first; r < rows; r += r_step) {
            const uint4 v = *reinterpret_cast<const uint4*>(park + r * FP4_PARK_LD + cg);
            const size_t tok = (size_t)(t0 + r);
            if (vec_ok) {
                uint4 o = v;
                if (p.R) {
                    const uint4 res = *reinterpret_cast<const uint4*>(p.R + tok * p.ldr + n0 + cg);
                    const uint32_t a[4] = {v.x, v.y, v.z, v.w}, b[4] = {res.x, res.y, res.z, res.w};
                    uint32_t cc[4];
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const __nv_bfloat162 pr = __halves2bfloat162(f2bf(bf_lo(a[j]) + bf_lo(b[j])), f2bf(bf_hi(a[j]) + bf_hi(b[j])));
                        cc[j] = *reinterpret_cast<const uint32_t*>(&pr);
                    }
                    o = make_uint4(cc[0], cc[1], cc[2], cc[3]);
                }
                *reinterpret_cast<uint4*>(cbase + tok * p.ldc + n0 + cg) = o;
            } else {
                const uint32_t a[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                for (int j = 0; j < 8; ++j)
                    if (n0 + cg + j < p.N) {
                        float y = (j & 1) ? bf_hi(a[j >> 1]) : bf_lo(a[j >> 1]);
                        if (p.R) y += bf2f(p.R[tok * p.ldr + n0 + cg + j]);
                        cbase[tok * p.ldc + n0 + cg + j] = f2bf(y);
                    }
            }
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 1) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(FP4_TMEM_COLS) : "memory");
    }
}

// Activation packer: bf16 [T][K] -> packed nibbles [Tpad][K/2] and scale atoms [Tpad/128][K/64][512] (Tpad = T rounded up to
// 128; the rows beyond T are written as zeros), the arithmetic of launch_quantize_nvfp4_lm_out.  One thread per 16 elements.
__global__ void __launch_bounds__(256) quantize_act_nvfp4_kernel(const bf16* __restrict__ x, int T, int K, uint8_t* __restrict__ packed,
                                                                 uint8_t* __restrict__ scales, long long total_blocks) {
    pdl_wait();
    const int bpr = K / 16;
    for (long long bid = (long long)blockIdx.x * blockDim.x + threadIdx.x; bid < total_blocks; bid += (long long)gridDim.x * blockDim.x) {
        const long long row = bid / bpr;
        const int sc = (int)(bid % bpr);
        uint32_t wd[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        if (row < T) {
            const uint4* src = reinterpret_cast<const uint4*>(x + row * K + sc * 16);
            const uint4 v0 = src[0], v1 = src[1];
            wd[0] = v0.x; wd[1] = v0.y; wd[2] = v0.z; wd[3] = v0.w; wd[4] = v1.x; wd[5] = v1.y; wd[6] = v1.z; wd[7] = v1.w;
        }
        const uint32_t lo4[4] = {wd[0], wd[1], wd[2], wd[3]}, hi4[4] = {wd[4], wd[5], wd[6], wd[7]};
        float inv;
        const uint8_t s8 = nvfp4_act_scale(fmaxf(nvfp4_amax8(lo4), nvfp4_amax8(hi4)), inv);
        *reinterpret_cast<uint2*>(packed + row * (K / 2) + sc * 8) = make_uint2(nvfp4_pack8(lo4, inv), nvfp4_pack8(hi4, inv));
        scales[nvfp4_scale_index(row, sc, K)] = s8;
    }
}

static bool fp4_tmap(CUtensorMap* tm, const void* ptr, long long rows, int k_bytes, int box_rows) {
    static PFN_cuTensorMapEncodeTiled_v12000 enc = nullptr;
    if (!enc) {
        cudaDriverEntryPointQueryResult qr;
        void* fn = nullptr;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &qr) != cudaSuccess || qr != cudaDriverEntryPointSuccess) return false;
        enc = (PFN_cuTensorMapEncodeTiled_v12000)fn;
    }
    const cuuint64_t dims[2] = {(cuuint64_t)k_bytes, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)k_bytes};
    const cuuint32_t box[2] = {128u, (cuuint32_t)box_rows};
    const cuuint32_t estr[2] = {1u, 1u};
    return enc(tm, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
               CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int T_TILE>
static int launch_fp4(const CUtensorMap& tmW, const CUtensorMap& tmA, const Fp4GemmParams& p, cudaStream_t stream) {
    static PerDeviceOnce attr;
    if (attr.pending()) {
        Q35_CUDA_OK(cudaFuncSetAttribute(gemm_nvfp4_tcgen05_kernel<T_TILE>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)fp4_smem(T_TILE)));
        attr.mark();
    }
    const dim3 grid((p.N + FP4_BM - 1) / FP4_BM, (p.T + T_TILE - 1) / T_TILE);
    if (g_pdl_launch) Q35_CUDA_OK(pdl_launch(gemm_nvfp4_tcgen05_kernel<T_TILE>, grid, dim3(FP4_THREADS), fp4_smem(T_TILE), stream, tmW, tmA, p));
    else gemm_nvfp4_tcgen05_kernel<T_TILE><<<grid, FP4_THREADS, fp4_smem(T_TILE), stream>>>(tmW, tmA, p);
    Q35_CUDA_OK(cudaGetLastError());
    g_launches.fetch_add(1);
    return QWEN35_OK;
}

}  // namespace q35

extern "C" size_t qwen35_b200_nvfp4_act_bytes(int tokens, int K, size_t* scales_bytes) {
    const size_t tpad = ((size_t)(tokens > 0 ? tokens : 0) + 127) / 128 * 128;
    if (scales_bytes) *scales_bytes = tpad / 128 * (size_t)(K / 64) * 512;
    return tpad * (size_t)(K / 2);
}

namespace q35 {

int quantize_act_nvfp4(const bf16* x, int tokens, int K, void* packed_out, void* scales_out, cudaStream_t stream) {
    if (!x || !packed_out || !scales_out || tokens <= 0 || K <= 0 || K % 64 != 0) {
        set_error("quantize_act_nvfp4: tokens (%d) > 0 and K (%d) a multiple of 64 required", tokens, K);
        return QWEN35_ERR_BAD_ARG;
    }
    const long long tpad = ((long long)tokens + 127) / 128 * 128, nblk = tpad * (K / 16);
    const int blocks = (int)((nblk + 255) / 256 < 148 * 16 ? (nblk + 255) / 256 : 148 * 16);
    Q35_CUDA_OK(pdl_launch(quantize_act_nvfp4_kernel, dim3(blocks), dim3(256), 0, stream, x, tokens, K, (uint8_t*)packed_out, (uint8_t*)scales_out, nblk));
    g_launches.fetch_add(1);
    return QWEN35_OK;
}

// n_rows: rows of the packed weight matrix (a multiple of 128: what the packer produced); n_out <= n_rows: output columns written
int gemm_nvfp4(const void* a_packed, const void* a_scales, int tokens, const void* w_packed, const void* w_scales, int n_rows, int n_out, int K,
               float alpha, void* C, int ldc, int out_f32, const bf16* R, int ldr, cudaStream_t stream) {
    if (!a_packed || !a_scales || !w_packed || !w_scales || !C || tokens <= 0 || n_rows <= 0 || n_rows % 128 != 0 || n_out <= 0 || n_out > n_rows ||
        K <= 0 || K % 256 != 0) {
        set_error("gemm_nvfp4: n_rows (%d) must be a multiple of 128 and K (%d) of 256, tokens (%d) > 0, 0 < n_out (%d) <= n_rows", n_rows, K, tokens, n_out);
        return QWEN35_ERR_BAD_ARG;
    }
    int* err = (int*)get_workspace();
    if (!err) return QWEN35_ERR_CUDA;
    const long long tpad = ((long long)tokens + 127) / 128 * 128;
    const int t_tile = tokens <= 16 ? 16 : tokens <= 32 ? 32 : tokens <= 64 ? 64 : 128;
    CUtensorMap tmW, tmA;
    if (!fp4_tmap(&tmW, w_packed, n_rows, K / 2, FP4_BM) || !fp4_tmap(&tmA, a_packed, tpad, K / 2, t_tile)) {
        set_error("gemm_nvfp4: tensor map creation failed (operands must be 16-byte aligned)");
        return QWEN35_ERR_CUDA;
    }
    Fp4GemmParams p{tokens, n_out, K, C, ldc, R, ldr, (const uint8_t*)w_scales, (const uint8_t*)a_scales, alpha, out_f32, err};
    switch (t_tile) {
        case 16: return launch_fp4<16>(tmW, tmA, p, stream);
        case 32: return launch_fp4<32>(tmW, tmA, p, stream);
        case 64: return launch_fp4<64>(tmW, tmA, p, stream);
        default: return launch_fp4<128>(tmW, tmA, p, stream);
    }
}

}  // namespace q35

extern "C" int qwen35_b200_quantize_act_nvfp4(const void* x, int tokens, int K, void* packed_out, void* scales_out, qwen35_stream_t stream) {
    return q35::quantize_act_nvfp4((const q35::bf16*)x, tokens, K, packed_out, scales_out, (cudaStream_t)stream);
}

extern "C" int qwen35_b200_gemm_nvfp4(const void* a_packed, const void* a_scales, int tokens, const void* w_packed, const void* w_scales, int n_rows,
                                      int K, float alpha, void* C, int ldc, int out_f32, const void* R, int ldr, qwen35_stream_t stream) {
    return q35::gemm_nvfp4(a_packed, a_scales, tokens, w_packed, w_scales, n_rows, n_rows, K, alpha, C, ldc, out_f32, (const q35::bf16*)R, ldr, (cudaStream_t)stream);
}
