// BF16 GEMM on the 5th-generation tensor cores (tcgen05 + TMEM) fed by TMA, for the prefill
// projections:  C[M,N] = A[M,K] . B[N,K]^T  with f32 accumulation in tensor memory.
//
// Replaces the cuBLAS calls of the reference's prefill (cublas_bf16_gemm, prefill.cu:895-903 and its
// ten call sites :1267-1434).  One CTA computes one 128 x 128 output tile:
//   warp 0     TMA producer: 128B-swizzled 64-wide K slices of A and B into a ring of stages
//   warp 1     allocates the TMEM columns, then one thread issues tcgen05.mma (M128 N128 K16 x4 per
//              stage) and commits each stage back to the producer
//   warps 2-5  tcgen05.ld the accumulator rows and park them as f32 in the idle stage buffers; then all six warps
//              read the tile back as row segments, round once to bf16 (what a bf16 linear layer returns), optionally
//              fuse the residual add or silu(gate)*up, and store 16 bytes per thread, a warp covering whole rows
// Six, three or two stages per CTA put one, two or three CTAs on an SM (the same bytes in flight per SM), chosen by the
// tile count so that no wave is left nearly empty and one tile's epilogue overlaps another's main loop.
// A skinny problem (M <= 128 rows of activations against a tall weight matrix) is bound by the fixed cost of a
// k-step (barrier hand-offs: about 0.3 us whatever the tile holds), not by bytes or flops, so it runs split along
// K: a thread-block cluster of S CTAs shares one 128 x 128 output tile, each CTA accumulates its slice of K in
// TMEM, parks the f32 tile in its own shared memory, and after a cluster barrier CTA r sums columns
// [r*128/S, (r+1)*128/S) over all peers through distributed shared memory (fixed order: deterministic) and
// applies the epilogue.  No partial sums go through global memory and no second kernel runs.
// Every wait is bounded; a wait that runs out sets the status word and the CTA unwinds normally.
#include <cuda.h>
#include <cstdlib>
#include <cuda_fp16.h>

#include "common.cuh"
#include "runtime.h"

namespace q35 {

constexpr int GEMM_BM = 128, GEMM_BN = 128, GEMM_BK = 64;
constexpr int GEMM_THREADS = 192;
constexpr uint32_t GEMM_STAGE_BYTES = (GEMM_BM + GEMM_BN) * GEMM_BK * 2;   // 32 KB
__host__ __device__ constexpr uint32_t gemm_stage_bytes(int bn) { return (uint32_t)(GEMM_BM + bn) * GEMM_BK * 2; }
// 6 stages for the wide problems (one CTA per SM); the skinny ones run a few k-steps per CTA: 3 stages, two CTAs per SM
constexpr int GEMM_STAGES_WIDE = 6, GEMM_STAGES_SKINNY = 3, GEMM_STAGES_THIRD = 2;     // one, two, three CTAs per SM
// the 64-column tile of the one-row-of-tiles problems (24 KB per stage): 8 stages for one CTA per SM, 4 for two
constexpr int GEMM_BN_NARROW = 64, GEMM_STAGES_NARROW = 8, GEMM_STAGES_NARROW_SPLIT = 4;
// The epilogue parks the f32 accumulator tile in the (then idle) stage buffers as [row][GEMM_PARK_LD]: with a pitch of
// 132 floats the float4 accesses of eight adjacent rows (writing, one row per thread) and of one row's adjacent column
// groups (reading) both spread over all 32 banks.
// The 256-column tile of the many-wave problems parks its accumulator rounded to bf16, [row][GEMM_PARK_LD_WIDE] (a pitch of
// 132 words: the 16-byte stores of eight adjacent rows cover all 32 banks); residual or SiLU * up are applied by the store pass.
constexpr int GEMM_BN_WIDE = 256, GEMM_STAGES_WIDE_TILE = 2, GEMM_PARK_LD_WIDE = GEMM_BN_WIDE + 8;
__host__ __device__ constexpr uint32_t gemm_park_bytes(int bn) {
    return bn == GEMM_BN_WIDE ? (uint32_t)GEMM_BM * GEMM_PARK_LD_WIDE * 2 : (uint32_t)GEMM_BM * (bn + 4) * 4;
}
__host__ __device__ constexpr uint32_t gemm_tile_bytes(int stages, int bn = GEMM_BN) {
    return stages * gemm_stage_bytes(bn) > gemm_park_bytes(bn) ? stages * gemm_stage_bytes(bn) : ((gemm_park_bytes(bn) + 1023u) & ~1023u);
}
__host__ __device__ constexpr uint32_t gemm_smem(int stages, int bn = GEMM_BN) { return gemm_tile_bytes(stages, bn) + 1024 /*align*/ + 256 /*barriers*/; }
// CTAs that fit an SM's 227 KB with this much dynamic shared memory each (1 KB reserved per CTA)
__host__ __device__ constexpr int gemm_ctas_per_sm(uint32_t smem) { return smem + 1024 <= 77 * 1024 ? 3 : (smem + 1024 <= 116 * 1024 ? 2 : 1); }
static_assert(GEMM_STAGES_SKINNY * GEMM_STAGE_BYTES >= GEMM_BM * GEMM_BN * 4, "the split-K form parks its f32 tile [column][row] in the stage buffers");
constexpr int GEMM_MAX_SPLIT = 8;        // portable cluster size
constexpr unsigned GEMM_SPIN_LIMIT = 20u * 1000u * 1000u;
enum GemmEpi { EPI_BF16 = 0, EPI_RESIDUAL = 1, EPI_SILU_MUL = 2 };

struct GemmParams {
    int M, N, K;            // N counts output columns
    bf16* C; int ldc;
    const bf16* R; int ldr; // residual (EPI_RESIDUAL)
    int up_row_offset;      // EPI_SILU_MUL: B row of "up" = up_row_offset + column
    int* err;
    int pdl_early;          // B is a constant weight matrix: load its first tiles in front of the dependency wait, release the successor early
};

__device__ __forceinline__ uint32_t g_smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ void g_mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void g_mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool g_mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok) : "r"(bar), "r"(parity) : "memory");
    return ok != 0;
}
// bounded wait; returns false (and records the error) when the limit is hit
__device__ __forceinline__ bool g_mbar_wait(uint32_t bar, uint32_t parity, int* err, volatile int* s_abort) {
    unsigned it = 0;
    while (!g_mbar_try_wait(bar, parity)) {
        if (*s_abort) return false;
        if (++it > GEMM_SPIN_LIMIT) { *s_abort = 1; atomicCAS(err, 0, (int)ERR_BARRIER_TIMEOUT); return false; }
    }
    return true;
}
__device__ __forceinline__ void g_tma_load_2d(uint32_t dst, const CUtensorMap* tm, int x, int y, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
        ::"r"(dst), "l"(tm), "r"(x), "r"(y), "r"(bar) : "memory");
}

// 64-bit shared-memory matrix descriptor, K-major operand, 128-byte swizzle:
// start address >> 4 | LBO (unused for this layout) | SBO = 1024 B between 8-row groups | version 1 | layout 2
__device__ __forceinline__ uint64_t make_smem_desc(uint32_t smem_addr) {
    uint64_t d = 0;
    d |= (uint64_t)((smem_addr & 0x3FFFFu) >> 4);
    d |= (uint64_t)1 << 16;
    d |= (uint64_t)(1024 >> 4) << 32;
    d |= (uint64_t)1 << 46;
    d |= (uint64_t)2 << 61;
    return d;
}
// instruction descriptor: D f32, A/B bf16, both K-major, N at [17,23) in units of 8, M at [24,29) in units of 16
__host__ __device__ constexpr uint32_t gemm_idesc(int bn) { return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(bn >> 3) << 17) | ((uint32_t)(GEMM_BM >> 4) << 24); }

__device__ __forceinline__ void umma_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate) : "memory");
}
// A operand in tensor memory (128 lanes = rows, one 32-bit column per two bf16 of K), B operand in shared memory
__device__ __forceinline__ void umma_bf16_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}"
        ::"r"(tmem_d), "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate) : "memory");
}
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&r)[8]) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};"
                 ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]) : "memory");
}
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr) : "memory");
}
__device__ __forceinline__ void umma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr) : "memory");
}

// ---- cluster helpers (split-K) ----
__device__ __forceinline__ uint32_t cluster_ctarank() { uint32_t r; asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r)); return r; }
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t map_to_cta(uint32_t local_smem_addr, uint32_t cta) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local_smem_addr), "r"(cta));
    return r;
}
__device__ __forceinline__ float ld_dsmem(uint32_t addr) {
    float v;
    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr));
    return v;
}

// epilogue arithmetic on 8 adjacent output columns of one row; acc = f32 sums (SILU: gate then up), one 16-byte store
template <int EPI>
__device__ __forceinline__ void epilogue_store8(const GemmParams& p, int row, int n, const float* g, const float* u) {
    float y[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        if (EPI == EPI_SILU_MUL) y[j] = rbf(silu_f(rbf(g[j]))) * rbf(u[j]);
        else y[j] = rbf(g[j]);
    }
    bf16* dst = p.C + (size_t)row * p.ldc + n;
    if (n + 8 <= p.N && ((reinterpret_cast<uintptr_t>(dst) & 15) == 0) && (EPI != EPI_RESIDUAL || ((reinterpret_cast<uintptr_t>(p.R + (size_t)row * p.ldr + n) & 15) == 0))) {
        if (EPI == EPI_RESIDUAL) {
            const uint4 r = *reinterpret_cast<const uint4*>(p.R + (size_t)row * p.ldr + n);
            y[0] += bf_lo(r.x); y[1] += bf_hi(r.x); y[2] += bf_lo(r.y); y[3] += bf_hi(r.y);
            y[4] += bf_lo(r.z); y[5] += bf_hi(r.z); y[6] += bf_lo(r.w); y[7] += bf_hi(r.w);
        }
        uint32_t o[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const __nv_bfloat162 pr = __halves2bfloat162(f2bf(y[2 * j]), f2bf(y[2 * j + 1]));
            o[j] = *reinterpret_cast<const uint32_t*>(&pr);
        }
        *reinterpret_cast<uint4*>(dst) = make_uint4(o[0], o[1], o[2], o[3]);
    } else {
#pragma unroll
        for (int j = 0; j < 8; ++j)
            if (n + j < p.N) {
                float v = y[j];
                if (EPI == EPI_RESIDUAL) v += bf2f(p.R[(size_t)row * p.ldr + n + j]);
                dst[j] = f2bf(v);
            }
    }
}

// Second half of the split-K epilogue: every CTA of the cluster has parked its f32 tile [column][row] at the same
// shared-memory offset; CTA `rank` finishes columns [rank * BN_OUT / S, +BN_OUT / S) for `rows` rows.  A work item is one
// row x 8 adjacent columns: all peers' values are requested before the first is used (one remote round trip, not S), then
// summed in peer order, so the result does not depend on timing.  `t` is the calling thread's index among `nt` workers.
template <int EPI, int BN = GEMM_BN, bool ROT = false>
__device__ __forceinline__ void cluster_reduce_store(const GemmParams& p, uint32_t park_local, int S, int rows, int m0, int n0, int t, int nt) {
    constexpr int BN_OUT = (EPI == EPI_SILU_MUL) ? BN / 2 : BN;
    const uint32_t rank = cluster_ctarank();
    // 8-column groups rank, rank + S, rank + 2S, ... of the tile belong to this CTA (any S up to the group count)
    const int my_groups = (BN_OUT / 8 - (int)rank + S - 1) / S;
    for (int item = t; item < rows * my_groups; item += nt) {
        const int r = item % rows, cg = item / rows;
        const int col = ((int)rank + cg * S) * 8;       // first of 8 output columns within the tile
        float g[8], u[8], v[GEMM_MAX_SPLIT][8];
#pragma unroll
        for (int peer = 0; peer < GEMM_MAX_SPLIT; ++peer)
            if (peer < S) {
                const uint32_t base = map_to_cta(park_local, (uint32_t)peer);
#pragma unroll
                for (int e = 0; e < 8; ++e) v[peer][e] = ld_dsmem(base + (uint32_t)(((col + e) * GEMM_BM + (ROT ? ((r + col + e) & 63) : r)) * 4));
            }
#pragma unroll
        for (int e = 0; e < 8; ++e) { g[e] = 0.f; u[e] = 0.f; }
#pragma unroll
        for (int peer = 0; peer < GEMM_MAX_SPLIT; ++peer)
            if (peer < S) {
#pragma unroll
                for (int e = 0; e < 8; ++e) g[e] += v[peer][e];
            }
        if (EPI == EPI_SILU_MUL) {
#pragma unroll
            for (int peer = 0; peer < GEMM_MAX_SPLIT; ++peer)
                if (peer < S) {
                    const uint32_t base = map_to_cta(park_local, (uint32_t)peer);
#pragma unroll
                    for (int e = 0; e < 8; ++e)
                        v[peer][e] = ld_dsmem(base + (uint32_t)(((BN / 2 + col + e) * GEMM_BM + (ROT ? ((r + BN / 2 + col + e) & 63) : r)) * 4));
                }
#pragma unroll
            for (int peer = 0; peer < GEMM_MAX_SPLIT; ++peer)
                if (peer < S) {
#pragma unroll
                    for (int e = 0; e < 8; ++e) u[e] += v[peer][e];
                }
        }
        epilogue_store8<EPI>(p, m0 + r, n0 + col, g, u);
    }
}

// The same store pass for a CTA on its own (no split): its tile is read with plain shared-memory loads (a
// ld.shared::cluster round trip costs several times more, and the SiLU form makes two of them in a row).  Layout as
// cluster_reduce_store<.., true> reads it: [column][GEMM_BM], the rows of column c rotated by c.
template <int EPI, int BN>
__device__ __forceinline__ void rotated_tile_store(const GemmParams& p, const float* park, int rows, int m0, int n0, int t, int nt) {
    constexpr int BN_OUT = (EPI == EPI_SILU_MUL) ? BN / 2 : BN;
    for (int item = t; item < rows * (BN_OUT / 8); item += nt) {
        const int r = item % rows, col = (item / rows) * 8;
        float g[8], u[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            g[e] = park[(col + e) * GEMM_BM + ((r + col + e) & 63)];
            u[e] = (EPI == EPI_SILU_MUL) ? park[(BN / 2 + col + e) * GEMM_BM + ((r + BN / 2 + col + e) & 63)] : 0.f;
        }
        epilogue_store8<EPI>(p, m0 + r, n0 + col, g, u);
    }
}

__device__ __forceinline__ float4 ld_smem4(uint32_t addr) {
    float4 v;
    asm volatile("ld.shared.v4.f32 {%0,%1,%2,%3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(addr) : "memory");
    return v;
}

// Store pass of a one-CTA tile over its parked accumulator [row][BN + 4].  A work item is one row x 8 adjacent
// output columns; consecutive threads take consecutive column groups of a row, so the 16-byte stores (and residual loads) of
// a warp cover whole row segments.  Four rows are in flight per thread: their loads are all issued before the first is used.
template <int EPI, int BN>
__device__ __forceinline__ void parked_tile_store(const GemmParams& p, uint32_t park_local, int rows, int m0, int n0, int t, int nt) {
    constexpr int BN_OUT = (EPI == EPI_SILU_MUL) ? BN / 2 : BN;
    constexpr int PARK_LD = BN + 4;
    constexpr int NG = BN_OUT / 8;
    constexpr int UNR = 4;
    const int col = (t % NG) * 8, r_first = t / NG, r_step = nt / NG;
    // the fast path: whole 16-byte groups inside N, both pointers 16-byte aligned for every row
    const bool vec_ok = n0 + col + 8 <= p.N && ((reinterpret_cast<uintptr_t>(p.C + n0 + col) | (size_t)p.ldc * 2) & 15) == 0 &&
                        (EPI != EPI_RESIDUAL || ((reinterpret_cast<uintptr_t>(p.R + n0 + col) | (size_t)p.ldr * 2) & 15) == 0);
    for (int rb = r_first; rb < rows; rb += UNR * r_step) {
        float g[UNR][8], u[UNR][8];
        uint4 res[UNR];
#pragma unroll
        for (int q = 0; q < UNR; ++q) {
            const int r = rb + q * r_step;
            res[q] = make_uint4(0u, 0u, 0u, 0u);
            if (EPI == EPI_RESIDUAL && vec_ok && r < rows) res[q] = *reinterpret_cast<const uint4*>(p.R + (size_t)(m0 + r) * p.ldr + n0 + col);
        }
#pragma unroll
        for (int q = 0; q < UNR; ++q) {
            const int r = min(rb + q * r_step, rows - 1);
            const uint32_t off = (uint32_t)((r * PARK_LD + col) * 4);
            const float4 a = ld_smem4(park_local + off), b = ld_smem4(park_local + off + 16);
            g[q][0] = a.x; g[q][1] = a.y; g[q][2] = a.z; g[q][3] = a.w; g[q][4] = b.x; g[q][5] = b.y; g[q][6] = b.z; g[q][7] = b.w;
#pragma unroll
            for (int e = 0; e < 8; ++e) u[q][e] = 0.f;
            if (EPI == EPI_SILU_MUL) {
                const float4 c = ld_smem4(park_local + off + BN * 2), d = ld_smem4(park_local + off + BN * 2 + 16);
                u[q][0] = c.x; u[q][1] = c.y; u[q][2] = c.z; u[q][3] = c.w; u[q][4] = d.x; u[q][5] = d.y; u[q][6] = d.z; u[q][7] = d.w;
            }
        }
#pragma unroll
        for (int q = 0; q < UNR; ++q) {
            const int r = rb + q * r_step;
            if (r >= rows) break;
            if (!vec_ok) { epilogue_store8<EPI>(p, m0 + r, n0 + col, g[q], u[q]); continue; }
            float y[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) y[j] = (EPI == EPI_SILU_MUL) ? rbf(silu_f(rbf(g[q][j]))) * rbf(u[q][j]) : rbf(g[q][j]);
            if (EPI == EPI_RESIDUAL) {
                y[0] += bf_lo(res[q].x); y[1] += bf_hi(res[q].x); y[2] += bf_lo(res[q].y); y[3] += bf_hi(res[q].y);
                y[4] += bf_lo(res[q].z); y[5] += bf_hi(res[q].z); y[6] += bf_lo(res[q].w); y[7] += bf_hi(res[q].w);
            }
            uint32_t o[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const __nv_bfloat162 pr = __halves2bfloat162(f2bf(y[2 * j]), f2bf(y[2 * j + 1]));
                o[j] = *reinterpret_cast<const uint32_t*>(&pr);
            }
            *reinterpret_cast<uint4*>(p.C + (size_t)(m0 + r) * p.ldc + n0 + col) = make_uint4(o[0], o[1], o[2], o[3]);
        }
    }
}

// Store pass of a 256-column tile over its parked bf16 results [row][GEMM_PARK_LD_WIDE]: a work item is one row x 8 adjacent
// output columns (16 bytes); consecutive threads take consecutive column groups of a row.  The residual is added here
// (rounded sum + residual, rounded again: the same arithmetic as the narrower tiles).
template <int EPI>
__device__ __forceinline__ void parked_tile_store_wide(const GemmParams& p, const bf16* park, int rows, int m0, int n0, int t, int nt) {
    constexpr int BN_OUT = (EPI == EPI_SILU_MUL) ? GEMM_BN_WIDE / 2 : GEMM_BN_WIDE;
    constexpr int NG = BN_OUT / 8;
    const int col = (t % NG) * 8, r_first = t / NG, r_step = nt / NG;
    const bool vec_ok = n0 + col + 8 <= p.N && ((reinterpret_cast<uintptr_t>(p.C + n0 + col) | (size_t)p.ldc * 2) & 15) == 0 &&
                        (EPI != EPI_RESIDUAL || ((reinterpret_cast<uintptr_t>(p.R + n0 + col) | (size_t)p.ldr * 2) & 15) == 0);
    for (int r = r_first; r < rows; r += r_step) {
        uint4 v = *reinterpret_cast<const uint4*>(park + (size_t)r * GEMM_PARK_LD_WIDE + col);
        if (EPI == EPI_SILU_MUL) {              // gate columns [0, 128), up columns [128, 256) of the parked row, both bf16 already
            const uint4 u = *reinterpret_cast<const uint4*>(park + (size_t)r * GEMM_PARK_LD_WIDE + GEMM_BN_WIDE / 2 + col);
            const uint32_t g4[4] = {v.x, v.y, v.z, v.w}, u4[4] = {u.x, u.y, u.z, u.w};
            uint32_t y4[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const __nv_bfloat162 pr = __halves2bfloat162(f2bf(rbf(silu_f(bf_lo(g4[j]))) * bf_lo(u4[j])), f2bf(rbf(silu_f(bf_hi(g4[j]))) * bf_hi(u4[j])));
                y4[j] = *reinterpret_cast<const uint32_t*>(&pr);
            }
            v = make_uint4(y4[0], y4[1], y4[2], y4[3]);
        }
        if (vec_ok) {
            uint4 o = v;
            if (EPI == EPI_RESIDUAL) {
                const uint4 res = *reinterpret_cast<const uint4*>(p.R + (size_t)(m0 + r) * p.ldr + n0 + col);
                const uint32_t a[4] = {v.x, v.y, v.z, v.w}, b[4] = {res.x, res.y, res.z, res.w};
                uint32_t c[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const __nv_bfloat162 pr = __halves2bfloat162(f2bf(bf_lo(a[j]) + bf_lo(b[j])), f2bf(bf_hi(a[j]) + bf_hi(b[j])));
                    c[j] = *reinterpret_cast<const uint32_t*>(&pr);
                }
                o = make_uint4(c[0], c[1], c[2], c[3]);
            }
            *reinterpret_cast<uint4*>(p.C + (size_t)(m0 + r) * p.ldc + n0 + col) = o;
        } else {
            const uint32_t a[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int j = 0; j < 8; ++j)
                if (n0 + col + j < p.N) {
                    float y = (j & 1) ? bf_hi(a[j >> 1]) : bf_lo(a[j >> 1]);
                    if (EPI == EPI_RESIDUAL) y += bf2f(p.R[(size_t)(m0 + r) * p.ldr + n0 + col + j]);
                    p.C[(size_t)(m0 + r) * p.ldc + n0 + col + j] = f2bf(y);
                }
        }
    }
}

// SPLIT: gridDim.z = cluster size S along K (1, 2, 4 or 8); the cluster shares one output tile.  BN: columns of the tile.
template <int EPI, int STAGES, bool SPLIT, int BN = GEMM_BN>
__global__ void __launch_bounds__(GEMM_THREADS, gemm_ctas_per_sm(gemm_smem(STAGES, BN)))
gemm_bf16_tcgen05_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, const GemmParams p) {
    extern __shared__ unsigned char g_smem_raw[];
    // 128B-swizzled tiles need 1024-byte alignment
    const uint32_t raw = g_smem_u32(g_smem_raw);
    const uint32_t tiles = (raw + 1023u) & ~1023u;
    unsigned char* tiles_ptr = g_smem_raw + (tiles - raw);
    uint64_t* bars = reinterpret_cast<uint64_t*>(tiles_ptr + gemm_tile_bytes(STAGES, BN));
    const uint32_t full0 = g_smem_u32(bars), empty0 = full0 + 8 * STAGES, tfull = empty0 + 8 * STAGES;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 1);
    volatile int* s_abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    constexpr int BN_OUT = (EPI == EPI_SILU_MUL) ? BN / 2 : BN;
    constexpr uint32_t SB = gemm_stage_bytes(BN);
    // the B tile arrives as one or two boxes of B_BOX weight rows: the second box holds the rows that follow, or (SiLU
    // epilogue) the up-projection rows that belong to the tile's gate rows
    constexpr int B_BOX = (BN == GEMM_BN) ? 64 : (BN == GEMM_BN_WIDE) ? 128 : (EPI == EPI_SILU_MUL ? BN / 2 : BN), B_NBOX = BN / B_BOX;
    const int n0 = blockIdx.x * BN_OUT, m0 = blockIdx.y * GEMM_BM;
    const int nkb_all = p.K / GEMM_BK;
    const int S = SPLIT ? (int)gridDim.z : 1, z = SPLIT ? (int)blockIdx.z : 0;
    const int kb_begin = (int)(((long long)z * nkb_all) / S), kb_end = (int)(((long long)(z + 1) * nkb_all) / S);
    const int nkb = kb_end - kb_begin;

    if (threadIdx.x == 0) {
        asm volatile("prefetch.tensormap [%0];" ::"l"(&tmA) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(&tmB) : "memory");
        *s_abort = 0;
        for (int i = 0; i < STAGES; ++i) { g_mbar_init(full0 + 8 * i, 1); g_mbar_init(empty0 + 8 * i, 1); }
        g_mbar_init(tfull, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(g_smem_u32(tmem_slot)), "r"((uint32_t)BN) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem_base = *tmem_slot;
    // Barriers, TMEM and tensor maps are set up.  What the predecessor wrote is touched only behind a pdl_wait(): by the copy
    // thread in front of its first activation tile, and by every thread in front of the store pass.
    if (p.pdl_early) pdl_trigger();

    if (warp == 0) {
        if (lane == 0) {
            // weight tiles of the first ring round: constants, so they may be under way while the predecessor still runs
            const int pre = p.pdl_early ? min(STAGES, nkb) : 0;
            for (int i = 0; i < pre; ++i) {
                const uint32_t b_dst = tiles + i * SB + GEMM_BM * GEMM_BK * 2;
                g_mbar_expect_tx(full0 + 8 * i, SB);
                g_tma_load_2d(b_dst, &tmB, (kb_begin + i) * GEMM_BK, n0, full0 + 8 * i);
                if (B_NBOX == 2)
                    g_tma_load_2d(b_dst + B_BOX * GEMM_BK * 2, &tmB, (kb_begin + i) * GEMM_BK, (EPI == EPI_SILU_MUL ? p.up_row_offset : B_BOX) + n0, full0 + 8 * i);
            }
            pdl_wait();
            int issued = pre;
            for (int i = 0; i < nkb; ++i) {
                const int st = i % STAGES, kb = kb_begin + i;
                const uint32_t a_dst = tiles + st * SB, b_dst = a_dst + GEMM_BM * GEMM_BK * 2;
                if (i >= pre) {
                    if (!g_mbar_wait(empty0 + 8 * st, ((i / STAGES) & 1) ^ 1, p.err, s_abort)) break;
                    g_mbar_expect_tx(full0 + 8 * st, SB);
                    g_tma_load_2d(b_dst, &tmB, kb * GEMM_BK, n0, full0 + 8 * st);
                    if (B_NBOX == 2)
                        g_tma_load_2d(b_dst + B_BOX * GEMM_BK * 2, &tmB, kb * GEMM_BK, (EPI == EPI_SILU_MUL ? p.up_row_offset : B_BOX) + n0, full0 + 8 * st);
                }
                g_tma_load_2d(a_dst, &tmA, kb * GEMM_BK, m0, full0 + 8 * st);
                issued = max(issued, i + 1);
            }
            // every copy this CTA issued must have landed before it may exit (matters only after an abort)
            if (*s_abort) {
                for (int i = max(0, issued - STAGES); i < issued; ++i) {
                    unsigned it = 0;
                    while (!g_mbar_try_wait(full0 + 8 * (i % STAGES), (i / STAGES) & 1) && ++it < GEMM_SPIN_LIMIT) {}
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            bool ok = true;
            for (int i = 0; i < nkb && ok; ++i) {
                const int st = i % STAGES;
                ok = g_mbar_wait(full0 + 8 * st, (i / STAGES) & 1, p.err, s_abort);
                if (!ok) break;
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const uint32_t a_addr = tiles + st * SB, b_addr = a_addr + GEMM_BM * GEMM_BK * 2;
                const uint64_t adesc = make_smem_desc(a_addr), bdesc = make_smem_desc(b_addr);
#pragma unroll
                for (int k = 0; k < GEMM_BK / 16; ++k)   // 32 bytes of K per instruction: advance the start-address field by 2
                    umma_bf16(tmem_base, adesc + (uint64_t)(2 * k), bdesc + (uint64_t)(2 * k), gemm_idesc(BN), (i > 0 || k > 0) ? 1u : 0u);
                umma_commit(empty0 + 8 * st);       // frees the stage when these MMAs have read it
            }
            umma_commit(tfull);                     // accumulator complete (also fires after an abort so the epilogue wakes)
        }
    } else {
        // ---- epilogue: warp w may touch TMEM lanes [32*(w%4), +32) ----
        const int q = warp & 3;
        const int rloc = q * 32 + lane;
        // warp-uniform, because tcgen05.ld is a warp-wide instruction
        const bool ok = __all_sync(0xffffffffu, g_mbar_wait(tfull, 0, p.err, s_abort) && !*s_abort);
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        if (BN == GEMM_BN_WIDE) {
            // 256-column tile: the accumulator rows are rounded to bf16 and parked; the store pass (all six warps) does the rest
            bf16* parkh = reinterpret_cast<bf16*>(tiles_ptr) + (size_t)rloc * GEMM_PARK_LD_WIDE;
            if (m0 + q * 32 < p.M) {
#pragma unroll 1
                for (int c = 0; c < BN / 32; ++c) {
                    uint32_t v[32];
                    if (ok) {
                        tmem_ld32(tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(c * 32), v);
                        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
                    }
#pragma unroll
                    for (int j = 0; j < 32; j += 8) {
                        uint32_t o[4];
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            const __nv_bfloat162 pr = __halves2bfloat162(f2bf(ok ? __uint_as_float(v[j + 2 * e]) : 0.f), f2bf(ok ? __uint_as_float(v[j + 2 * e + 1]) : 0.f));
                            o[e] = *reinterpret_cast<const uint32_t*>(&pr);
                        }
                        *reinterpret_cast<uint4*>(parkh + c * 32 + j) = make_uint4(o[0], o[1], o[2], o[3]);
                    }
                }
            }
        } else {
        // park the f32 tile in the (now idle) stage buffers.  Split K: column-major [column][row], which makes the peers'
        // reads through distributed shared memory whole 128-byte lines (measured faster there than 16-byte pieces of rows);
        // one CTA per tile: row-major with a padded pitch, read back below as row segments.
        float* park = reinterpret_cast<float*>(tiles_ptr);
        if (m0 + q * 32 < p.M) {                                // else: rows of this warp are never read back
#pragma unroll
            for (int c = 0; c < BN / 32; ++c) {
                uint32_t v[32];
                if (ok) {
                    tmem_ld32(tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(c * 32), v);
                    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
                }
                if (SPLIT) {
#pragma unroll
                    for (int j = 0; j < 32; ++j) park[(c * 32 + j) * GEMM_BM + rloc] = ok ? __uint_as_float(v[j]) : 0.f;
                } else {
#pragma unroll
                    for (int j = 0; j < 32; j += 4)
                        *reinterpret_cast<float4*>(park + rloc * (BN + 4) + c * 32 + j) =
                            ok ? make_float4(__uint_as_float(v[j]), __uint_as_float(v[j + 1]), __uint_as_float(v[j + 2]), __uint_as_float(v[j + 3]))
                               : make_float4(0.f, 0.f, 0.f, 0.f);
                }
            }
        }
        }
    }
    __syncwarp();
    pdl_wait();
    if (SPLIT) {
        // every thread of every CTA of the cluster passes both barriers, whatever happened above
        cluster_sync_all();
        if (warp >= 2 && !*s_abort)
            cluster_reduce_store<EPI, BN>(p, tiles, S, min(GEMM_BM, p.M - m0), m0, n0, (int)threadIdx.x - 64, GEMM_THREADS - 64);
        __syncwarp();
        cluster_sync_all();                                     // no CTA leaves while a peer may still read its tile
    } else {
        // the store pass is arithmetic and address work on shared memory: all six warps take part (the copy and MMA warps
        // are idle by now)
        __syncthreads();
        if (!*s_abort) {
            if (BN == GEMM_BN_WIDE) parked_tile_store_wide<EPI>(p, reinterpret_cast<const bf16*>(tiles_ptr), min(GEMM_BM, p.M - m0), m0, n0, (int)threadIdx.x, GEMM_THREADS);
            else parked_tile_store<EPI, BN>(p, tiles, min(GEMM_BM, p.M - m0), m0, n0, (int)threadIdx.x, GEMM_THREADS);
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 1) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"((uint32_t)BN) : "memory");
    }
}

// ------------------------------------------------------------------------------------------------------------
// Q4_K weights: C[M <= 64, N] = epi(A[M, K] . dequant(W[N, K])^T).  Same split-K cluster scheme as above, but the
// weight operand never exists as bf16 in global OR shared memory: the dequantised tile goes straight into tensor memory
// and is the MMA's A operand (128 weight rows = 128 lanes; the activation rows are the N dimension, read from shared
// memory).  The form before this one wrote the bf16 tile into shared memory for the MMA to read back: its counters
// showed the shared-memory data pipe full in the main loop (1 060 wavefronts per k-step = the k-step's cycles: 362
// tile stores, 384 MMA operand reads, 115 raw loads, 200 of TMA writes); this form needs about 440.
//   warp 0      TMA producer of the activation tiles (two 64-wide slabs per 128-wide k-step, 64 token rows each)
//   warp 18     TMA producer of the RAW Q4_K super-blocks, one box of 144 bytes x 64 rows per half tile (a whole
//               super-block row per request: HBM sees contiguous 144-byte pieces, never 16- or 32-byte ones); its own
//               warp so that the raw ring runs its full depth ahead of the dequantisation
//   warps 2-17  dequantise from the raw ring into tensor memory: warp w owns the lanes 32 (w % 4) .. + 31 (the only ones
//               it may touch), thread = one weight row; eight warps take the even k-steps, eight the odd ones, a thread
//               converting one 64-weight group (four 8-column tcgen05.st) per super-block
//   warps 1, 19 MMA issue: 8 x (M128 N<=64 K16) per k-step once both operands of the stage are there.  Two issuing
//               threads, one for the even k-steps and one for the odd ones, each with an accumulator of its own (the
//               epilogue adds them): with the operands ready, ONE thread needs ~0.5 us per k-step to get its barrier
//               observations and 8 instructions through, and the whole main loop ran at that pace; two threads took the
//               27B tree verify from 12.0 to 10.5 ms
//   warps 2-17  epilogue afterwards (park, cluster reduce, store); the accumulator is [weight row][token]
// The weight operand is value = fma_bf16(q, bf16(d*sc), -bf16(dmin*m)), two weights per instruction: the published f32
// dequantisation (d*sc)*q - dmin*m followed by a rounding to bf16 cost ~10 instructions per weight on the CUDA cores.
// qwen35_b200_dequant_q4k keeps the published arithmetic bit for bit.  (An f16 weight operand beside bf16 activations
// is not an option: kind::f16 with different A and B formats raised "illegal instruction" on this GPU.)
constexpr int Q4K_THREADS = 640;                                // 2 + 16 dequantisation warps + the raw producer + the second MMA issuer
constexpr int Q4K_DQ_WARPS = 16;
constexpr int Q4K_RAW_WARP = 2 + Q4K_DQ_WARPS, Q4K_MMA2_WARP = Q4K_RAW_WARP + 1;
constexpr int Q4K_STAGES = 4, Q4K_RAW_STAGES = 3;
constexpr uint32_t Q4K_X_SLAB = 64 * 128;                                              // bytes: 64 token rows x 64 k
constexpr uint32_t Q4K_STAGE_BYTES = 2 * Q4K_X_SLAB;                                  // 16 KB of activations per 128-wide k-step
constexpr uint32_t Q4K_RAW_BYTES = 128 * 144;                                          // one super-block per tile row
// tensor memory: per stage 64 columns of weights (128 k as bf16 pairs), then two f32 accumulators [128 weights][64 tokens]
constexpr uint32_t Q4K_W_COLS = 64, Q4K_D_COL = Q4K_STAGES * Q4K_W_COLS, Q4K_TMEM_COLS = 512;
static_assert(Q4K_D_COL + 2 * 64 <= Q4K_TMEM_COLS, "tensor memory budget");
__device__ __forceinline__ uint32_t q4k_idesc(int n_tokens) {      // D f32, A and B bf16, M = 128 weight rows, N = tokens rounded up to 16
    return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n_tokens >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
}
constexpr uint32_t Q4K_SMEM_USED = Q4K_STAGES * Q4K_STAGE_BYTES + Q4K_RAW_STAGES * Q4K_RAW_BYTES + 1024 + 256;
// The CTA takes all 512 tensor-memory columns of its SM, so no other tensor-memory kernel may share the SM with it: a CTA of
// another stream's GEMM that blocks in tcgen05.alloc beside it while its own cluster waits for it at a cluster barrier could
// close a cycle with this kernel's cluster (tree verify runs a small bf16 GEMM beside a Q4_K projection).  Asking for 200 KB
// of shared memory leaves room for no kernel of this library that allocates tensor memory (the smallest needs 49 KB).
constexpr uint32_t Q4K_SMEM = Q4K_SMEM_USED > 200u * 1024u ? Q4K_SMEM_USED : 200u * 1024u;
static_assert(Q4K_STAGES * Q4K_STAGE_BYTES >= GEMM_BM * GEMM_BN * 4, "the parked f32 tile reuses the stage buffers");

__device__ __forceinline__ void q4k_scale_min_u32(uint32_t s0, uint32_t s1, uint32_t s2, int j, float& sc, float& mn) {
    // s0, s1, s2 = scale bytes 0-3, 4-7, 8-11
    const uint32_t bj = (j < 4) ? (s0 >> (8 * j)) & 0xFF : (s1 >> (8 * (j - 4))) & 0xFF;          // scales[j]
    if (j < 4) {
        const uint32_t bj4 = (s1 >> (8 * j)) & 0xFF;                                                // scales[j+4]
        sc = (float)(bj & 63); mn = (float)(bj4 & 63);
    } else {
        const uint32_t bj4 = (s2 >> (8 * (j - 4))) & 0xFF;                                          // scales[j+4]
        const uint32_t bjm = (s0 >> (8 * (j - 4))) & 0xFF;                                          // scales[j-4]
        sc = (float)((bj4 & 0xF) | ((bjm >> 6) << 4)); mn = (float)((bj4 >> 4) | ((bj >> 6) << 4));
    }
}

template <int EPI>
__global__ void __launch_bounds__(Q4K_THREADS, 1)
gemm_q4k_tcgen05_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmW, const GemmParams p) {
    constexpr int STAGES = Q4K_STAGES, RS = Q4K_RAW_STAGES;
    extern __shared__ unsigned char g_smem_raw[];
    const uint32_t raw = g_smem_u32(g_smem_raw);
    const uint32_t tiles = (raw + 1023u) & ~1023u;
    unsigned char* tiles_ptr = g_smem_raw + (tiles - raw);
    unsigned char* rawring_ptr = tiles_ptr + STAGES * Q4K_STAGE_BYTES;
    const uint32_t rawring = tiles + STAGES * Q4K_STAGE_BYTES;
    uint64_t* bars = reinterpret_cast<uint64_t*>(rawring_ptr + RS * Q4K_RAW_BYTES);
    const uint32_t fulla0 = g_smem_u32(bars), fullb0 = fulla0 + 8 * STAGES, empty0 = fullb0 + 8 * STAGES, fullr0 = empty0 + 8 * STAGES,
                   emptyr0 = fullr0 + 8 * RS, tfull = emptyr0 + 8 * RS;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 3 * STAGES + 2 * RS + 1);
    volatile int* s_abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    constexpr int BN_OUT = (EPI == EPI_SILU_MUL) ? GEMM_BN / 2 : GEMM_BN;
    const int n0 = blockIdx.x * BN_OUT;
    const int sb_all = p.K / 256;
    const int S = (int)gridDim.z, z = (int)blockIdx.z;
    const int sb_begin = (int)(((long long)z * sb_all) / S), sb_end = (int)(((long long)(z + 1) * sb_all) / S);
    const int nk2 = 2 * (sb_end - sb_begin);                 // 128-wide k-steps of this CTA (two per super-block)

    if (threadIdx.x == 0) {
        asm volatile("prefetch.tensormap [%0];" ::"l"(&tmA) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(&tmW) : "memory");
        *s_abort = 0;
        for (int i = 0; i < STAGES; ++i) { g_mbar_init(fulla0 + 8 * i, 1); g_mbar_init(fullb0 + 8 * i, Q4K_DQ_WARPS / 2); g_mbar_init(empty0 + 8 * i, 1); }
        for (int i = 0; i < RS; ++i) { g_mbar_init(fullr0 + 8 * i, 1); g_mbar_init(emptyr0 + 8 * i, Q4K_DQ_WARPS); }
        g_mbar_init(tfull, 2);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(g_smem_u32(tmem_slot)), "r"(Q4K_TMEM_COLS) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem_base = *tmem_slot;
    pdl_trigger();
    // No pdl_wait() here: the weights are constants, so the raw producer and the dequantisation warps start at once and have
    // the first stages of weights in tensor memory while the kernel in front of this one is still running (when that kernel
    // lets its successor in early).  What the predecessor writes is touched only behind a pdl_wait(): the activation loads
    // below, and the store pass (every thread waits in front of it).

    if (warp == 0) {
        // activation tiles: k-step i may be issued as soon as the MMAs of k-step i - STAGES have read the stage
        if (lane == 0) {
            pdl_wait();
            int issued_a = 0;
            for (int i = 0; i < nk2; ++i) {
                const int st = i % STAGES;
                if (!g_mbar_wait(empty0 + 8 * st, ((i / STAGES) & 1) ^ 1, p.err, s_abort)) break;
                g_mbar_expect_tx(fulla0 + 8 * st, 2 * Q4K_X_SLAB);
                const uint32_t a_dst = tiles + st * Q4K_STAGE_BYTES;
                const int kcol = (sb_begin * 2 + i) * 128;
                g_tma_load_2d(a_dst, &tmA, kcol, 0, fulla0 + 8 * st);
                g_tma_load_2d(a_dst + Q4K_X_SLAB, &tmA, kcol + 64, 0, fulla0 + 8 * st);
                issued_a = i + 1;
            }
            if (*s_abort) {      // copies in flight must land before the CTA may exit
                for (int i = max(0, issued_a - STAGES); i < issued_a; ++i) {
                    unsigned it = 0;
                    while (!g_mbar_try_wait(fulla0 + 8 * (i % STAGES), (i / STAGES) & 1) && ++it < GEMM_SPIN_LIMIT) {}
                }
            }
        }
    } else if (warp == Q4K_RAW_WARP) {
        // raw super-blocks, a producer of their own: a slot is refilled the moment both k-steps of its super-block are
        // dequantised, RS super-blocks ahead of the consumers, whatever the state of the activation ring (issued from the
        // activation producer's loop, a refill waited for that loop's stage and ran barely one k-step ahead of its use)
        if (lane == 0) {
            int issued_r = 0;
            const int nsb = sb_end - sb_begin;
            for (int j = 0; j < nsb; ++j) {
                const int rs = j % RS;
                if (!g_mbar_wait(emptyr0 + 8 * rs, ((j / RS) & 1) ^ 1, p.err, s_abort)) break;
                g_mbar_expect_tx(fullr0 + 8 * rs, Q4K_RAW_BYTES);
                const uint32_t dst = rawring + rs * Q4K_RAW_BYTES;
                g_tma_load_2d(dst, &tmW, (sb_begin + j) * 144, n0, fullr0 + 8 * rs);
                g_tma_load_2d(dst + 64 * 144, &tmW, (sb_begin + j) * 144, (EPI == EPI_SILU_MUL ? p.up_row_offset : 64) + n0, fullr0 + 8 * rs);
                issued_r = j + 1;
            }
            if (*s_abort) {
                for (int j = max(0, issued_r - RS); j < issued_r; ++j) {
                    unsigned it = 0;
                    while (!g_mbar_try_wait(fullr0 + 8 * (j % RS), (j / RS) & 1) && ++it < GEMM_SPIN_LIMIT) {}
                }
            }
        }
    } else if (warp == 1 || warp == Q4K_MMA2_WARP) {
        if (lane == 0) {
            const uint32_t idesc = q4k_idesc(min(64, max(16, (p.M + 15) & ~15)));
            const int who = (warp == 1) ? 0 : 1;                  // k-steps who, who + 2, ... into accumulator `who` (nk2 is even)
            const uint32_t acc = tmem_base + Q4K_D_COL + 64u * (uint32_t)who;
            for (int i = who; i < nk2; i += 2) {
                const int st = i % STAGES;
                if (!g_mbar_wait(fulla0 + 8 * st, (i / STAGES) & 1, p.err, s_abort)) break;
                if (!g_mbar_wait(fullb0 + 8 * st, (i / STAGES) & 1, p.err, s_abort)) break;
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const uint32_t x_addr = tiles + st * Q4K_STAGE_BYTES, w_col = tmem_base + (uint32_t)st * Q4K_W_COLS;
#pragma unroll
                for (int sl = 0; sl < 2; ++sl) {
                    const uint64_t xdesc = make_smem_desc(x_addr + sl * Q4K_X_SLAB);
#pragma unroll
                    for (int k = 0; k < 4; ++k)      // 16 k = 8 columns of the weight operand, 32 bytes of the activation rows
                        umma_bf16_ts(acc, w_col + (uint32_t)(sl * 32 + k * 8), xdesc + (uint64_t)(2 * k), idesc, (i > who || sl > 0 || k > 0) ? 1u : 0u);
                }
                umma_commit(empty0 + 8 * st);
            }
            umma_commit(tfull);
        }
    } else {
        // ---- dequantisation: thread (row, h, par) converts group g = 2*par + h of every super-block (32 nibble bytes = 64
        // weights = slab h of k-step `par`): half of the warps work on the even k-steps, half on the odd ones, so the 6-bit
        // scales of a group are decoded once and a warp meets the barriers once per 64 weights. ----
        const int dw = warp - 2, row = (warp & 3) * 32 + lane, h = (dw >> 2) & 1, par = dw >> 3;
        const int sh = 16 * h;
        // slab h of the stage: columns 32 h + k / 2; the low nibbles are k = 0..31 of the slab, the high ones k = 32..63
        const uint32_t wdst = tmem_base + ((uint32_t)((warp & 3) * 32) << 16) + (uint32_t)(32 * h);
        const unsigned char* const rbase = rawring_ptr + row * 144 + 16 + 32 * (2 * par + h);
        const __nv_bfloat162 k128 = __float2bfloat162_rn(128.0f);
        int rs = 0;
        uint32_t rs_par = 0;
        const int nsb = sb_end - sb_begin;
        bool alive = true;
        for (int j = 0; j < nsb && alive; ++j) {
            alive = __all_sync(0xffffffffu, g_mbar_wait(fullr0 + 8 * rs, rs_par, p.err, s_abort));
            if (!alive) break;
            const unsigned char* rb = rawring_ptr + row * 144 + rs * Q4K_RAW_BYTES;
            const uint4 hd = *reinterpret_cast<const uint4*>(rb);
            const uint4 qa = *reinterpret_cast<const uint4*>(rbase + rs * Q4K_RAW_BYTES);
            const uint4 qb = *reinterpret_cast<const uint4*>(rbase + rs * Q4K_RAW_BYTES + 16);
            const __half2 dd = *reinterpret_cast<const __half2*>(&hd.x);
            const float d = __low2float(dd), ndmin = -__high2float(dd);
            const uint32_t sx = hd.y >> sh, sy = hd.z >> sh, sz = hd.w >> sh;      // scale bytes 2h.., 4+2h.., 8+2h..
            uint32_t sc0, mn0, sc1, mn1;                                            // sub-blocks 2g and 2g+1 of group g = 2*par + h
            if (par == 0) {
                sc0 = sx & 63u; sc1 = (sx >> 8) & 63u; mn0 = sy & 63u; mn1 = (sy >> 8) & 63u;
            } else {
                sc0 = (sz & 0xFu) | ((sx >> 2) & 0x30u);         mn0 = ((sz >> 4) & 0xFu) | ((sy >> 2) & 0x30u);
                sc1 = ((sz >> 8) & 0xFu) | ((sx >> 10) & 0x30u); mn1 = ((sz >> 12) & 0xFu) | ((sy >> 10) & 0x30u);
            }
            // operand value = bf16 fma(q, bf16(d*sc), -bf16(dmin*m)): d*sc and dmin*m are exact in f32 (11 + 6 bits), one
            // rounding each to bf16 (round-to-nearest is symmetric, so the sign goes in before it), then one fused rounding
            const __nv_bfloat162 ds0 = __float2bfloat162_rn(__fmul_rn(d, (float)sc0)), ds1 = __float2bfloat162_rn(__fmul_rn(d, (float)sc1));
            const __nv_bfloat162 nm0 = __float2bfloat162_rn(__fmul_rn(ndmin, (float)mn0)), nm1 = __float2bfloat162_rn(__fmul_rn(ndmin, (float)mn1));
            const uint32_t w[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
            const int i = 2 * j + par, st = i % STAGES;                            // this warp's k-step and its stage
            alive = __all_sync(0xffffffffu, g_mbar_wait(empty0 + 8 * st, ((i / STAGES) & 1) ^ 1, p.err, s_abort));
            if (!alive) break;
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");       // the MMAs that read this stage are done
#pragma unroll
            for (int hi = 0; hi < 2; ++hi) {                        // 32 weights from the low nibbles, then 32 from the high ones
                const __nv_bfloat162 dsx = hi ? ds1 : ds0, nmx = hi ? nm1 : nm0;
#pragma unroll
                for (int half = 0; half < 2; ++half) {
                    uint32_t o[8];
#pragma unroll
                    for (int h2 = 0; h2 < 4; ++h2) {
                        const uint32_t word = w[4 * half + h2];
                        const uint32_t nib = (hi ? (word >> 4) : word) & 0x0F0F0F0Fu;
                        // bytes (q, 0x43) are the bf16 numbers 128 + q: exact, no integer conversion
                        const uint32_t u01 = __byte_perm(nib, 0x43004300u, 0x7150), u23 = __byte_perm(nib, 0x43004300u, 0x7352);
                        const __nv_bfloat162 x01 = __hsub2(*reinterpret_cast<const __nv_bfloat162*>(&u01), k128);
                        const __nv_bfloat162 x23 = __hsub2(*reinterpret_cast<const __nv_bfloat162*>(&u23), k128);
                        const __nv_bfloat162 y01 = __hfma2(x01, dsx, nmx), y23 = __hfma2(x23, dsx, nmx);
                        o[2 * h2] = *reinterpret_cast<const uint32_t*>(&y01);
                        o[2 * h2 + 1] = *reinterpret_cast<const uint32_t*>(&y23);
                    }
                    tmem_st8(wdst + (uint32_t)(st * (int)Q4K_W_COLS + 16 * hi + 8 * half), o);   // the pair's first weight in the low half
                }
            }
            asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
            asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
            __syncwarp();
            if (lane == 0) {
                asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(fullb0 + 8 * st) : "memory");
                asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(emptyr0 + 8 * rs) : "memory");   // this warp is done with the super-block
            }
            if (++rs == RS) { rs = 0; rs_par ^= 1u; }
        }
        {
            // ---- epilogue part 1: park the f32 tile in the idle stage buffers; the four warps of a lane quarter take 16
            // tokens each ----
            const int wrow = (warp & 3) * 32 + lane;                    // this thread's weight row = its tensor-memory lane
            const int tok0 = (dw >> 2) * 16;
            const bool ok = __all_sync(0xffffffffu, g_mbar_wait(tfull, 0, p.err, s_abort) && !*s_abort);
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            // [weight row of the tile][token], the tokens of row w rotated by w so that a warp's stores (32 rows, one token)
            // fall into 32 different banks; cluster_reduce_store<.., true> undoes the rotation
            float* park = reinterpret_cast<float*>(tiles_ptr) + wrow * GEMM_BM;
            if (tok0 < p.M) {                                           // tokens that do not exist are never read back
                uint32_t v[16];
                if (ok) {
                    uint32_t v2[16];
                    const uint32_t src = tmem_base + Q4K_D_COL + ((uint32_t)((warp & 3) * 32) << 16) + (uint32_t)tok0;
                    tmem_ld16(src, v);
                    tmem_ld16(src + 64u, v2);
                    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
                    for (int j = 0; j < 16; ++j) v[j] = __float_as_uint(__uint_as_float(v[j]) + __uint_as_float(v2[j]));
                }
#pragma unroll
                for (int j = 0; j < 16; ++j) park[(tok0 + j + wrow) & 63] = ok ? __uint_as_float(v[j]) : 0.f;
            }
        }
    }
    __syncwarp();
    pdl_wait();
    // every thread of every CTA of the cluster passes these barriers, whatever happened above; a CTA on its own (no split)
    // needs neither the cluster's barrier nor the second one (nobody else reads its tile)
    if (S > 1) cluster_sync_all(); else __syncthreads();
    if (warp >= 2 && !*s_abort) {
        if (S > 1) cluster_reduce_store<EPI, GEMM_BN, true>(p, tiles, S, min(64, p.M), 0, n0, (int)threadIdx.x - 64, Q4K_THREADS - 64);
        else rotated_tile_store<EPI, GEMM_BN>(p, reinterpret_cast<const float*>(tiles_ptr), min(64, p.M), 0, n0, (int)threadIdx.x - 64, Q4K_THREADS - 64);
    }
    __syncwarp();
    if (S > 1) cluster_sync_all();
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 1) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(Q4K_TMEM_COLS) : "memory");
    }
}

// ---------------------------------------- host side -------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*, const cuuint64_t*,
                                  const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult qres;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &qres) == cudaSuccess && qres == cudaDriverEntryPointSuccess)
            fn = (EncodeTiledFn)p;
    }
    return fn;
}

// 2-D bf16 tensor [rows, cols] with row stride `ld` elements; box = 64 columns x box_rows, 128-byte swizzle.
// (also used by the batched-decode attention for its K / V pages)
bool make_tmap(CUtensorMap* tm, const void* ptr, int rows, int cols, int ld, int box_rows) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
    cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    return fn(tm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// bf16 tensor of rank 2 or 3 (dims innermost first, strides in bytes for dims 1..), 128-byte swizzle: the inner box extent
// must be 64 elements.  Used by the attention kernels for their Q / K / V^T boxes.
bool make_tmap_bf16(CUtensorMap* tm, const void* ptr, int rank, const unsigned long long* dims, const unsigned long long* strides_bytes,
                    const unsigned* box) {
    EncodeTiledFn fn = encode_fn();
    if (!fn || rank < 2 || rank > 3) return false;
    cuuint64_t d[3], st[2];
    cuuint32_t b[3], estr[3] = {1, 1, 1};
    for (int i = 0; i < rank; ++i) { d[i] = dims[i]; b[i] = box[i]; }
    for (int i = 0; i + 1 < rank; ++i) st[i] = strides_bytes[i];
    return fn(tm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, (cuuint32_t)rank, const_cast<void*>(ptr), d, st, b, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Q4_K super-blocks as a 2-D byte tensor [rows][K/256 * 144]; box = one super-block (144 bytes) x 64 rows, no swizzle.
static bool make_tmap_q4k(CUtensorMap* tm, const void* ptr, int rows, int K) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return false;
    const cuuint64_t row_bytes = (cuuint64_t)(K / 256) * 144;
    cuuint64_t dims[2] = {row_bytes, (cuuint64_t)rows};
    cuuint64_t strides[1] = {row_bytes};
    cuuint32_t box[2] = {144, 64};
    cuuint32_t estr[2] = {1, 1};
    return fn(tm, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(ptr), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// plain (non-cluster) launch of a GEMM kernel; joins a programmatic-dependent-launch chain when the caller asked for it
template <typename K>
static cudaError_t gemm_launch(K kernel, dim3 grid, size_t smem, cudaStream_t stream, const CUtensorMap& tmA, const CUtensorMap& tmB, const GemmParams& p) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid; cfg.blockDim = dim3(GEMM_THREADS); cfg.dynamicSmemBytes = smem; cfg.stream = stream;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at; cfg.numAttrs = g_pdl_launch ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, tmA, tmB, p);
}

template <int E, int ST, int BN = GEMM_BN>
static int gemm_plain(dim3 grid, cudaStream_t stream, const CUtensorMap& tmA, const CUtensorMap& tmB, const GemmParams& p) {
    static PerDeviceOnce attr;
    if (attr.pending()) {
        Q35_CUDA_OK(cudaFuncSetAttribute(gemm_bf16_tcgen05_kernel<E, ST, false, BN>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)gemm_smem(ST, BN)));
        attr.mark();
    }
    Q35_CUDA_OK(gemm_launch(gemm_bf16_tcgen05_kernel<E, ST, false, BN>, grid, gemm_smem(ST, BN), stream, tmA, tmB, p));
    return QWEN35_OK;
}
template <int ST, int BN = GEMM_BN>
static int gemm_plain_epi(int epi, dim3 grid, cudaStream_t stream, const CUtensorMap& tmA, const CUtensorMap& tmB, const GemmParams& p) {
    switch (epi) {
        case EPI_BF16: return gemm_plain<EPI_BF16, ST, BN>(grid, stream, tmA, tmB, p);
        case EPI_RESIDUAL: return gemm_plain<EPI_RESIDUAL, ST, BN>(grid, stream, tmA, tmB, p);
        default: return gemm_plain<EPI_SILU_MUL, ST, BN>(grid, stream, tmA, tmB, p);
    }
}
// split-K over a cluster of `split` CTAs along grid z
template <int E, int ST, int BN>
static int gemm_split(dim3 grid, int split, cudaStream_t stream, const CUtensorMap& tmA, const CUtensorMap& tmB, const GemmParams& p) {
    static PerDeviceOnce attr;
    if (attr.pending()) {
        Q35_CUDA_OK(cudaFuncSetAttribute(gemm_bf16_tcgen05_kernel<E, ST, true, BN>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)gemm_smem(ST, BN)));
        attr.mark();
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid.x, grid.y, split);
    cfg.blockDim = dim3(GEMM_THREADS);
    cfg.dynamicSmemBytes = gemm_smem(ST, BN);
    cfg.stream = stream;
    cudaLaunchAttribute at[2];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = 1; at[0].val.clusterDim.y = 1; at[0].val.clusterDim.z = (unsigned)split;
    at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at; cfg.numAttrs = g_pdl_launch ? 2 : 1;
    Q35_CUDA_OK(cudaLaunchKernelEx(&cfg, gemm_bf16_tcgen05_kernel<E, ST, true, BN>, tmA, tmB, p));
    return QWEN35_OK;
}
template <int ST, int BN>
static int gemm_split_epi(int epi, dim3 grid, int split, cudaStream_t stream, const CUtensorMap& tmA, const CUtensorMap& tmB, const GemmParams& p) {
    switch (epi) {
        case EPI_BF16: return gemm_split<EPI_BF16, ST, BN>(grid, split, stream, tmA, tmB, p);
        case EPI_RESIDUAL: return gemm_split<EPI_RESIDUAL, ST, BN>(grid, split, stream, tmA, tmB, p);
        default: return gemm_split<EPI_SILU_MUL, ST, BN>(grid, split, stream, tmA, tmB, p);
    }
}

// C[M,N] (row stride ldc) = epi(A[M,K] (row stride lda) . B[*,K]^T).  epi: 0 bf16, 1 + R, 2 silu(gate)*up with
// gate rows [0,N) and up rows [up_row_offset, up_row_offset+N) of B.  b_rows = number of rows of B.
int gemm_bf16(const bf16* A, int lda, const bf16* B, int b_rows, bf16* C, int ldc, const bf16* R, int ldr,
              int M, int N, int K, int epi, int up_row_offset, cudaStream_t stream) {
    if (M <= 0 || N <= 0) return QWEN35_OK;
    if (K % GEMM_BK != 0 || (lda % 8) != 0 || ((uintptr_t)A & 15) || ((uintptr_t)B & 15)) {
        set_error("gemm_bf16: K must be a multiple of 64 and operands 16-byte aligned");
        return QWEN35_ERR_BAD_ARG;
    }
    void* ws = get_workspace();
    if (!ws) return QWEN35_ERR_CUDA;
    if (epi < 0 || epi > 2) { set_error("gemm_bf16: unknown epilogue %d", epi); return QWEN35_ERR_BAD_ARG; }
    // Many rows of 256-column tiles whose count is a little above a whole number of waves (296 tiles, two CTAs per SM): the
    // last, nearly empty wave costs as much as a full one.  The rows of tiles that spill over are split off into a call of
    // their own (the 4096 x 7168 gate/up GEMM: 896 tiles = 3 waves + 8 tiles; 31 rows of tiles fill 2.93 waves, the 32nd runs
    // as a 128-row problem behind them).
    {
        const int mt = (M + GEMM_BM - 1) / GEMM_BM;
        const int ntw = (N + ((epi == EPI_SILU_MUL) ? GEMM_BN_WIDE / 2 : GEMM_BN_WIDE) - 1) / ((epi == EPI_SILU_MUL) ? GEMM_BN_WIDE / 2 : GEMM_BN_WIDE);
        const int over = (mt * ntw) % 296;
        if (epi != EPI_RESIDUAL && mt >= 9 && mt * ntw > 296 && over > 0 && over <= 45) {
            const int peel = (over + ntw - 1) / ntw;
            if (peel * 4 <= mt) {
                const int m_main = (mt - peel) * GEMM_BM;
                const int st0 = gemm_bf16(A, lda, B, b_rows, C, ldc, R, ldr, m_main, N, K, epi, up_row_offset, stream);
                if (st0 != QWEN35_OK) return st0;
                return gemm_bf16(A + (size_t)m_main * lda, lda, B, b_rows, C + (size_t)m_main * ldc, ldc, R ? R + (size_t)m_main * ldr : nullptr, ldr,
                                 M - m_main, N, K, epi, up_row_offset, stream);
            }
        }
    }
    GemmParams p{M, N, K, C, ldc, R, ldr, up_row_offset, (int*)ws, g_pdl_early ? 1 : 0};
    const int nkb = K / GEMM_BK;
    const int m_tiles = (M + GEMM_BM - 1) / GEMM_BM;
    const int bn_out = (epi == EPI_SILU_MUL) ? GEMM_BN / 2 : GEMM_BN;
    const int n_tiles = (N + bn_out - 1) / bn_out, tiles_total = m_tiles * n_tiles;
    CUtensorMap tmA, tmB;
    // One row of tiles that cannot fill the SMs with 128-column tiles (M <= 128: decode batches, tree nodes, draft rows, short
    // prompts): 64-column tiles double the CTA count, so the wide projections need no split along K at all (no cluster
    // barriers, no reduction through distributed shared memory) and the narrow ones reduce half as much.  A k-step costs
    // its barrier hand-offs whatever the tile holds, so the narrow tile is taken only where it does not lengthen a long k loop.
    const int bn_out_n = (epi == EPI_SILU_MUL) ? GEMM_BN_NARROW / 2 : GEMM_BN_NARROW;
    const int nt_n = (N + bn_out_n - 1) / bn_out_n;
    int split_n = 1, split_w = 1;
    while (split_n < GEMM_MAX_SPLIT && nt_n * split_n < 100 && nkb / (split_n * 2) >= 2) split_n *= 2;
    while (split_w < GEMM_MAX_SPLIT && n_tiles * split_w < 120 && nkb / (split_w * 2) >= 2) split_w *= 2;
    bool narrow = m_tiles == 1 && n_tiles < 148 && (split_n == 1 || nkb <= 16 || nkb / split_n <= nkb / split_w);
    // A few rows of tiles with long K (the out / down projections of a 1024-token prompt: 64 tiles of 128 columns): where the
    // 128-column tiles with their split leave SMs without a CTA, 64-column tiles with the same rule fill them (4.33 -> 4.19 ms
    // for the 1024-token prompt), and so they do where the wide form would need 8-CTA clusters and they need 4 (260 tokens:
    // 2.30 -> 2.23 ms); where the wide form already has a CTA per SM with clusters of 4 it stays (520 tokens: 160 CTAs either
    // way, and the wide form is the faster one there).
    int m_rows_n = 1;
    if (!narrow && m_tiles > 1 && tiles_total < 100 && nkb >= 16) {
        int sw = 1, sp = 1;
        while (sw < GEMM_MAX_SPLIT && tiles_total * sw < 120 && nkb / (sw * 2) >= 2) sw *= 2;
        while (sp < GEMM_MAX_SPLIT && nt_n * m_tiles * sp < 148 && nkb / (sp * 2) >= 2) sp *= 2;
        if (sp >= 2 && ((tiles_total * sw < 148 && nt_n * m_tiles * sp > tiles_total * sw) || (sw >= 8 && sp < sw))) { narrow = true; split_n = sp; m_rows_n = m_tiles; }
    }
    // Many waves of tiles (long prompts x wide matrices): the 128 x 128 tile reads 32 KB from L2 per 128 x 128 x 64 step, and the
    // SM's L2 port, shared by its two CTAs, is what bounds it.  A 128 x 256 tile reads 48 KB for twice the work (two CTAs of two
    // stages per SM, 256 tensor-memory columns each).
    const int bn_out_wd = (epi == EPI_SILU_MUL) ? GEMM_BN_WIDE / 2 : GEMM_BN_WIDE;
    const int nt_wd = (N + bn_out_wd - 1) / bn_out_wd;
    // Taken from 8 rows of tiles on, when its waves (two CTAs per SM) cost less than the 128-column tile's: a wave of the wide
    // tile takes 1.5-1.8 x as long for twice the work (measured at 4096 x 8224 x 1024 and 4096 x 7168 x 1024; the factor 1.5 was the
    // best of 1.2 / 1.5 / 1.8 over prompts of 1024 to 4096 tokens), and either form pays for a whole last wave.
    const int slots_n = tiles_total <= 148 ? 148 : (tiles_total > 296 && tiles_total <= 444) ? 444 : 296;
    const int waves_n = (tiles_total + slots_n - 1) / slots_n, waves_wd = (m_tiles * nt_wd + 295) / 296;
    const bool wide_tile = !narrow && epi != EPI_RESIDUAL && m_tiles >= 8 && 15 * waves_wd < 10 * waves_n;
    const int b_box = wide_tile ? 128 : !narrow ? 64 : (epi == EPI_SILU_MUL ? GEMM_BN_NARROW / 2 : GEMM_BN_NARROW);
    if (!make_tmap(&tmA, A, M, K, lda, GEMM_BM) || !make_tmap(&tmB, B, b_rows, K, K, b_box)) {
        set_error("cuTensorMapEncodeTiled failed (A %p [%d x %d] ld %d; B %p [%d x %d])", (const void*)A, M, K, lda, (const void*)B, b_rows, K);
        return QWEN35_ERR_CUDA;
    }
    int st = QWEN35_OK;
    if (wide_tile) {
        st = gemm_plain_epi<GEMM_STAGES_WIDE_TILE, GEMM_BN_WIDE>(epi, dim3(nt_wd, m_tiles), stream, tmA, tmB, p);
    } else if (narrow) {
        if (split_n == 1) st = gemm_plain_epi<GEMM_STAGES_NARROW, GEMM_BN_NARROW>(epi, dim3(nt_n, 1), stream, tmA, tmB, p);
        else st = gemm_split_epi<GEMM_STAGES_NARROW_SPLIT, GEMM_BN_NARROW>(epi, dim3(nt_n, m_rows_n), split_n, stream, tmA, tmB, p);
    } else {
        // a grid that cannot fill the SMs (few tiles, long K) splits K over clusters
        const bool small_grid = tiles_total < 100 && nkb >= 8;
        int split = 1;
        if (small_grid) while (split < GEMM_MAX_SPLIT && tiles_total * split < 120 && nkb / (split * 2) >= 2) split *= 2;
        const dim3 grid(n_tiles, m_tiles);
        // One CTA per SM with six stages while the tiles fit one wave; more tiles than SMs: three (two) stages per CTA let
        // two (three) CTAs share an SM -- the same bytes in flight per SM -- so that the prologue and epilogue of one tile
        // overlap the main loop of another and a tile count a little above a multiple of 148 does not leave a second wave
        // nearly empty.  Beyond three waves' worth of tiles the two-per-SM form is used.
        if (split > 1) st = gemm_split_epi<GEMM_STAGES_SKINNY, GEMM_BN>(epi, grid, split, stream, tmA, tmB, p);
        else if (m_tiles > 1 && tiles_total <= 148) st = gemm_plain_epi<GEMM_STAGES_WIDE>(epi, grid, stream, tmA, tmB, p);
        else if (tiles_total > 296 && tiles_total <= 444) st = gemm_plain_epi<GEMM_STAGES_THIRD>(epi, grid, stream, tmA, tmB, p);
        else st = gemm_plain_epi<GEMM_STAGES_SKINNY>(epi, grid, stream, tmA, tmB, p);
    }
    if (st != QWEN35_OK) return st;
    Q35_CUDA_OK(cudaGetLastError());
    g_launches.fetch_add(1);
    return QWEN35_OK;
}


// C[M, N] (M <= 64) = epi(A[M, K] . dequant(W)^T), W = Q4_K super-blocks [w_rows][K/256][144]; epi as gemm_bf16
// (epi 2: gate rows [0, N), up rows [up_row_offset, up_row_offset + N)).  K must be a multiple of 256.
int gemm_q4k(const bf16* A, int lda, const uint8_t* W, int w_rows, bf16* C, int ldc, const bf16* R, int ldr,
             int M, int N, int K, int epi, int up_row_offset, cudaStream_t stream) {
    if (M <= 0 || N <= 0) return QWEN35_OK;
    if (M > 64 || K % 256 != 0 || (lda % 8) != 0 || ((uintptr_t)A & 15) || ((uintptr_t)W & 15) || epi < 0 || epi > 2) {
        set_error("gemm_q4k: needs M <= 64, K a multiple of 256, 16-byte aligned operands, epilogue 0..2");
        return QWEN35_ERR_BAD_ARG;
    }
    void* ws = get_workspace();
    if (!ws) return QWEN35_ERR_CUDA;
    CUtensorMap tmA, tmW;
    if (!make_tmap(&tmA, A, M, K, lda, 64) || !make_tmap_q4k(&tmW, W, w_rows, K)) {
        set_error("cuTensorMapEncodeTiled failed (A %p [%d x %d] ld %d; W %p [%d rows])", (const void*)A, M, K, lda, (const void*)W, w_rows);
        return QWEN35_ERR_CUDA;
    }
    GemmParams qp{M, N, K, C, ldc, R, ldr, up_row_offset, (int*)ws, 0};
    const int bn_out = (epi == EPI_SILU_MUL) ? GEMM_BN / 2 : GEMM_BN;
    const int n_tiles = (N + bn_out - 1) / bn_out, nsb = K / 256;
    // one CTA per SM: the largest split (cluster size, not necessarily a power of two) that keeps the whole grid in ONE
    // wave, with at least 2 super-blocks per CTA.  (Doubling until "about full" put 40-tile shapes at 160 CTAs: a second
    // wave for 12 of them doubled the time.)
    static int sm_count = 0;
    if (!sm_count) {
        int dev = 0;
        Q35_CUDA_OK(cudaGetDevice(&dev));
        Q35_CUDA_OK(cudaDeviceGetAttribute(&sm_count, cudaDevAttrMultiProcessorCount, dev));
    }
    int split = sm_count / n_tiles;
    if (split > GEMM_MAX_SPLIT) split = GEMM_MAX_SPLIT;
    if (split < 1) split = 1;
    while (split > 1 && nsb / split < 2) --split;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(n_tiles, 1, split);
    cfg.blockDim = dim3(Q4K_THREADS);
    cfg.dynamicSmemBytes = Q4K_SMEM;
    cfg.stream = stream;
    cudaLaunchAttribute at[2];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = 1; at[0].val.clusterDim.y = 1; at[0].val.clusterDim.z = (unsigned)split;
    at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at; cfg.numAttrs = g_pdl_launch ? 2 : 1;
#define Q35_GEMM_Q4K(E)                                                                                                            \
    case E: {                                                                                                                      \
        static PerDeviceOnce attr;                                                                                                  \
        if (attr.pending()) {                                                                                                               \
            Q35_CUDA_OK(cudaFuncSetAttribute(gemm_q4k_tcgen05_kernel<E>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)Q4K_SMEM)); \
            attr.mark();                                                                                                           \
        }                                                                                                                          \
        Q35_CUDA_OK(cudaLaunchKernelEx(&cfg, gemm_q4k_tcgen05_kernel<E>, tmA, tmW, qp));                                                 \
        break;                                                                                                                     \
    }
    switch (epi) { Q35_GEMM_Q4K(EPI_BF16) Q35_GEMM_Q4K(EPI_RESIDUAL) Q35_GEMM_Q4K(EPI_SILU_MUL) }
#undef Q35_GEMM_Q4K
    Q35_CUDA_OK(cudaGetLastError());
    g_launches.fetch_add(1);
    return QWEN35_OK;
}

}  // namespace q35

extern "C" int qwen35_b200_gemm_q4k(const void* A, int lda, const void* W, int w_rows, void* C, int ldc, const void* R, int ldr,
                                    int M, int N, int K, int epilogue, int up_row_offset, qwen35_stream_t stream) {
    return q35::gemm_q4k((const q35::bf16*)A, lda, (const uint8_t*)W, w_rows, (q35::bf16*)C, ldc, (const q35::bf16*)R, ldr, M, N, K, epilogue, up_row_offset,
                         (cudaStream_t)stream);
}

extern "C" int qwen35_b200_gemm_bf16(const void* A, int lda, const void* B, int b_rows, void* C, int ldc, const void* R, int ldr,
                                     int M, int N, int K, int epilogue, int up_row_offset, qwen35_stream_t stream) {
    return q35::gemm_bf16((const q35::bf16*)A, lda, (const q35::bf16*)B, b_rows, (q35::bf16*)C, ldc, (const q35::bf16*)R, ldr,
                          M, N, K, epilogue, up_row_offset, (cudaStream_t)stream);
}
