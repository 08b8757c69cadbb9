// Causal GQA attention of the prompt pass on the 5th-generation tensor cores (tcgen05 + TMEM), operands by TMA.
//
// Replaces the reference's prefill attention (pf_causal_attn, models/qwen35_0p8b/prefill.cu:489-552, one warp per
// (query, head) on the CUDA cores).  Rounding points are those of the bf16 HuggingFace model: scores = bf16(q.k)/16,
// softmax in f32 over the whole row, P rounded to bf16, out = bf16(P.V), times bf16(sigmoid(gate)).
//
// One CTA = 32 queries x the 4 q heads of one kv head = 128 rows (row r: query r/4, head r%4) = the M side of every MMA.
//   warp 0     TMA producer: the Q tile once (a 3-D box: 64 dims x 4 heads x 32 tokens lands as 128 rows of 128 bytes), then
//              per 64-key chunk the K rows [64][256] and, in pass 2, the chunk of V^T [256 dims][64 keys]
//   warp 1     one thread issues tcgen05.mma: S[128 x 64] = Q K^T (16 instructions of K = 16), and in pass 2
//              O[128 x 256] += P V (4 instructions, B = the V^T rows, so every operand is K-major with 128-byte swizzle:
//              the layout of the GEMM in gemm_tcgen05.cu)
//   warps 2-9  softmax: two threads per row (32 keys of a chunk each); tcgen05.ld brings the scores into registers, so
//              maximum, normaliser and the P values need no shuffles.  Softmax over the whole row in two passes over the causal key range: pass 1 the
//              running row maximum and normaliser; pass 2 recomputes the same scores (same instructions, same values), writes
//              P = bf16(exp(s - m) / l) as the swizzled A operand of P.V (exp as 2^x on the special-function unit, the
//              division as a product with 1 / l).  At the end the O row comes from TMEM, is rounded,
//              gated and stored.
// V^T is a scratch copy of the layer's V rows made by att_transpose_v_kernel (64 x 64 tiles through shared memory).
// Every wait is bounded; a wait that runs out sets the status word and the CTA unwinds normally (TMEM is freed).
#include <cuda.h>
#include <cuda_fp16.h>

#include "common.cuh"
#include "runtime.h"

namespace q35 {

bool make_tmap_bf16(CUtensorMap* tm, const void* ptr, int rank, const unsigned long long* dims, const unsigned long long* strides_bytes,
                    const unsigned* box);      // gemm_tcgen05.cu

constexpr int AT_Q = 32, AT_ROWS = AT_Q * FA_GQA, AT_KEYS = 64;
constexpr int AT_THREADS = 320;            // copy warp, MMA warp, eight softmax warps
constexpr uint32_t AT_Q_BYTES = AT_ROWS * FA_HEAD_DIM * 2;          // 64 KB: four 16 KB blocks of 64 dims
constexpr uint32_t AT_K_BYTES = AT_KEYS * FA_HEAD_DIM * 2;          // 32 KB: four 8 KB blocks of 64 dims
constexpr uint32_t AT_V_BYTES = FA_HEAD_DIM * AT_KEYS * 2;          // 32 KB: 256 rows (dims) x 128 bytes (64 keys)
constexpr uint32_t AT_P_BYTES = AT_ROWS * AT_KEYS * 2;              // 16 KB
constexpr uint32_t AT_SMEM = 1024 + AT_Q_BYTES + 2 * AT_K_BYTES + 2 * AT_V_BYTES + 2 * AT_P_BYTES + 256;
constexpr unsigned AT_SPIN_LIMIT = 20u * 1000u * 1000u;
constexpr uint32_t AT_TMEM_COLS = 512, AT_TMEM_S = 256;              // O in columns [0, 256), two S buffers in [256, 384)

__device__ __forceinline__ bool at_wait(uint32_t bar, uint32_t parity, int* err, volatile int* s_abort) {
    unsigned it = 0;
    while (!mbar_try_wait(bar, parity)) {
        if (*s_abort) return false;
        if (++it > AT_SPIN_LIMIT) { *s_abort = 1; atomicCAS(err, 0, (int)ERR_BARRIER_TIMEOUT); return false; }
    }
    return true;
}
__device__ __forceinline__ void at_tma_3d(uint32_t dst, const void* tm, int x, int y, int z, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];"
        ::"r"(dst), "l"(tm), "r"(x), "r"(y), "r"(z), "r"(bar) : "memory");
}
// K-major operand, 128-byte swizzle, 1024 bytes between 8-row groups (the descriptor of gemm_tcgen05.cu)
__device__ __forceinline__ uint64_t at_desc(uint32_t smem_addr) {
    uint64_t d = 0;
    d |= (uint64_t)((smem_addr & 0x3FFFFu) >> 4);
    d |= (uint64_t)1 << 16;
    d |= (uint64_t)(1024 >> 4) << 32;
    d |= (uint64_t)1 << 46;
    d |= (uint64_t)2 << 61;
    return d;
}
__host__ __device__ constexpr uint32_t at_idesc(int n) { return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(AT_ROWS >> 4) << 24); }
__device__ __forceinline__ void at_mma(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate) : "memory");
}
__device__ __forceinline__ void at_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
// 2^x on the special-function unit (2 ulp).  The softmax weights are rounded to bf16 right after, so the approximation moves
// about one weight in 10^4 by a last place: the size of the effect the summation order of any GEMM has on its outputs.  The
// exact expf / division of the mma.sync kernels cost 25 instructions per score and made the softmax warps, not the tensor
// pipe, the bound of this kernel.
__device__ __forceinline__ float at_exp2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
constexpr float AT_LOG2E = 1.4426950408889634f;

__device__ __forceinline__ void at_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr) : "memory");
}

// V rows [kv head][position][256] -> V^T [kv head][256][s_pad] (positions >= S zero): 64 x 64 tiles through shared memory
__global__ void __launch_bounds__(256) att_transpose_v_kernel(const bf16* __restrict__ v_cache, bf16* __restrict__ vt, int S, int s_pad, int max_seq) {
    pdl_wait();
    __shared__ bf16 tile[64][66];
    const int t0 = blockIdx.x * 64, d0 = blockIdx.y * 64, kvh = blockIdx.z, tid = threadIdx.x;
    for (int i = tid; i < 64 * 32; i += 256) {
        const int ti = i / 32, dp = (i % 32) * 2;
        uint32_t v = 0u;
        if (t0 + ti < S) v = *reinterpret_cast<const uint32_t*>(v_cache + ((size_t)kvh * max_seq + t0 + ti) * FA_HEAD_DIM + d0 + dp);
        *reinterpret_cast<uint32_t*>(&tile[ti][dp]) = v;
    }
    __syncthreads();
    for (int i = tid; i < 64 * 32; i += 256) {
        const int di = i / 32, tp = (i % 32) * 2;
        const __nv_bfloat162 pr = __halves2bfloat162(tile[tp][di], tile[tp + 1][di]);
        *reinterpret_cast<__nv_bfloat162*>(vt + ((size_t)kvh * FA_HEAD_DIM + d0 + di) * s_pad + t0 + tp) = pr;
    }
}

struct AttParams {
    const bf16* proj; int ldp;      // gate of head h of token t: proj[t * ldp + h * 512 + 256 + d]
    bf16* out;                      // [S][2048]
    int S, max_seq;
    int* err;
};

__global__ void __launch_bounds__(AT_THREADS, 1)
attention_tcgen05_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmVT,
                         const AttParams p) {
    extern __shared__ unsigned char at_smem_raw[];
    const uint32_t raw = smem_u32(at_smem_raw), base = (raw + 1023u) & ~1023u;
    unsigned char* base_p = at_smem_raw + (base - raw);
    const uint32_t q_s = base, k_s = q_s + AT_Q_BYTES, v_s = k_s + 2 * AT_K_BYTES, p_s = v_s + 2 * AT_V_BYTES;
    unsigned char* p_ptr = base_p + AT_Q_BYTES + 2 * AT_K_BYTES + 2 * AT_V_BYTES;
    u64* bars = reinterpret_cast<u64*>(p_ptr + 2 * AT_P_BYTES);
    // barriers: 0 qfull | 1-4 full | 5-8 empty (ring of four 32 KB chunk buffers) | 9,10 sfull | 11,12 sfree | 13,14 pfull | 15,16 pfree | 17 ofull
    // K and V^T chunks share one ring: the copies are numbered in the order they are issued -- K(0) .. K(n-1) of pass 1, then
    // K(0), V(0), K(1), V(1), ... of pass 2 -- and copy L lands in buffer L mod 4, so pass 1 runs four chunks ahead of the MMAs
    // and pass 2 two.
    // The score accumulator and the P tile are double buffered: Q K^T of item i + 1 is issued before P V of item i, so the tensor
    // pipe works on the next scores while the softmax warps are busy with the current ones.
    const uint32_t bar0 = smem_u32(bars);
    auto B = [&](int i) { return bar0 + 8u * (uint32_t)i; };
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 18);
    volatile int* s_abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int blk = (int)gridDim.x - 1 - (int)blockIdx.x;          // long blocks first
    const int kvh = blockIdx.y, q0 = blk * AT_Q;
    const int t_last = min(q0 + AT_Q, p.S) - 1;
    const int nchunks = t_last / AT_KEYS + 1;

    if (threadIdx.x == 0) {
        asm volatile("prefetch.tensormap [%0];" ::"l"(&tmQ) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(&tmK) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(&tmVT) : "memory");
        *s_abort = 0;
        for (int i = 0; i < 18; ++i) mbar_init(B(i), (i >= 11 && i <= 14) ? 8u : 1u);    // sfree / pfull: one arrival per softmax warp
        mbar_fence_init();
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)), "r"(AT_TMEM_COLS) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem_base = *tmem_slot;
    pdl_wait();

    if (warp == 0) {
        if (lane == 0) {
            // Q tile: four boxes of 64 dims x 4 heads x 32 tokens
            mbar_arrive_expect_tx(B(0), AT_Q_BYTES);
            for (int db = 0; db < 4; ++db) at_tma_3d(q_s + db * (AT_ROWS * 128), &tmQ, db * 64, kvh * FA_GQA, q0, B(0));
            int L = 0;
            bool ok = true;
            for (int item = 0; item < 2 * nchunks && ok; ++item) {
                const int pass = item >= nchunks, c = pass ? item - nchunks : item;
                for (int part = 0; part <= pass && ok; ++part, ++L) {          // part 0: K chunk; part 1 (pass 2): V^T chunk
                    const int bf = L & 3;
                    ok = at_wait(B(5 + bf), ((L >> 2) & 1) ^ 1, p.err, s_abort);
                    if (!ok) break;
                    mbar_arrive_expect_tx(B(1 + bf), AT_K_BYTES);
                    if (part == 0) {
                        for (int db = 0; db < 4; ++db)
                            tma_load_2d(k_s + bf * AT_K_BYTES + db * (AT_KEYS * 128), &tmK, db * 64, kvh * p.max_seq + c * AT_KEYS, B(1 + bf));
                    } else {
                        tma_load_2d(k_s + bf * AT_K_BYTES, &tmVT, c * AT_KEYS, kvh * FA_HEAD_DIM, B(1 + bf));
                    }
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            bool ok = at_wait(B(0), 0, p.err, s_abort);
            const int nitems = 2 * nchunks;
            for (int step = 0; step <= nitems && ok; ++step) {
                if (step < nitems) {
                    // ---- S[step & 1] = Q K^T of item `step` ----
                    const int item = step, sb = item & 1, use = item >> 1;
                    const int L = item < nchunks ? item : nchunks + 2 * (item - nchunks), st = L & 3;
                    ok = at_wait(B(1 + st), (L >> 2) & 1, p.err, s_abort);
                    if (ok && use > 0) ok = at_wait(B(11 + sb), (use - 1) & 1, p.err, s_abort);      // the scores two items back have been read
                    if (!ok) break;
                    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
#pragma unroll
                    for (int db = 0; db < 4; ++db) {
                        const uint64_t adesc = at_desc(q_s + db * (AT_ROWS * 128)), bdesc = at_desc(k_s + st * AT_K_BYTES + db * (AT_KEYS * 128));
#pragma unroll
                        for (int k = 0; k < 4; ++k)
                            at_mma(tmem_base + AT_TMEM_S + sb * AT_KEYS, adesc + (uint64_t)(2 * k), bdesc + (uint64_t)(2 * k), at_idesc(AT_KEYS), (db > 0 || k > 0) ? 1u : 0u);
                    }
                    at_commit(B(5 + st));        // buffer free when these MMAs have read it
                    at_commit(B(9 + sb));        // scores ready
                }
                if (step - 1 >= nchunks) {
                    // ---- O += P V of the previous item (a pass-2 item) ----
                    const int c = step - 1 - nchunks, pb = c & 1, use = c >> 1;
                    const int L = nchunks + 2 * c + 1, vs = L & 3;
                    ok = at_wait(B(1 + vs), (L >> 2) & 1, p.err, s_abort) && at_wait(B(13 + pb), use & 1, p.err, s_abort);    // V^T chunk in, P written
                    if (!ok) break;
                    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                    const uint64_t adesc = at_desc(p_s + pb * AT_P_BYTES), bdesc = at_desc(k_s + vs * AT_K_BYTES);
#pragma unroll
                    for (int k = 0; k < 4; ++k)
                        at_mma(tmem_base, adesc + (uint64_t)(2 * k), bdesc + (uint64_t)(2 * k), at_idesc(FA_HEAD_DIM), (c > 0 || k > 0) ? 1u : 0u);
                    at_commit(B(5 + vs));        // buffer free
                    at_commit(B(15 + pb));       // P tile free
                }
            }
            at_commit(B(17));                // output complete (also fires after an abort so the softmax warps wake)
        }
    } else {
        // ---- softmax warps: warp w may touch TMEM lanes [32 (w % 4), +32).  Two threads per row: warps 2-5 take the first 32
        // keys of a chunk (and the first 128 output dimensions), warps 6-9 the other half, so each sub-partition has two warps
        // to interleave.  In pass 1 a thread keeps the maximum and normaliser of its own keys; the pair is merged once, through
        // shared memory, before pass 2. ----
        const int qd = warp & 3, half = (warp - 2) >> 2, r = qd * 32 + lane;
        const int t = q0 + r / FA_GQA, head = kvh * FA_GQA + r % FA_GQA;
        const uint32_t trow = tmem_base + ((uint32_t)(qd * 32) << 16);
        const bool live = t < p.S;
        float m = -INFINITY, l = 0.f;
        bool ok = true;
        float2* ml_x = reinterpret_cast<float2*>(p_ptr);       // [half][row]: the (idle) P tiles carry the exchange after pass 1
        for (int pass_i = 0; pass_i < 2; ++pass_i) {
        if (pass_i == 1) {
            // merge the two halves of every row.  Every softmax thread executes these two barriers exactly once, whatever
            // happened in pass 1, and no P tile is written before the second one.
            ml_x[half * AT_ROWS + r] = make_float2(m, l);
            asm volatile("bar.sync 1, 256;" ::: "memory");
            const float2 other = ml_x[(half ^ 1) * AT_ROWS + r];
            asm volatile("bar.sync 1, 256;" ::: "memory");
            const float n = fmaxf(m, other.x);
            l = (m == -INFINITY ? 0.f : l * at_exp2((m - n) * AT_LOG2E)) + (other.x == -INFINITY ? 0.f : other.y * at_exp2((other.x - n) * AT_LOG2E));
            m = n;
        }
        for (int item = pass_i * nchunks; item < (pass_i + 1) * nchunks && ok; ++item) {
            const int pass = pass_i, c = pass ? item - nchunks : item, j0 = c * AT_KEYS + half * 32;
            const int sb = item & 1;
            ok = __all_sync(0xffffffffu, ok && at_wait(B(9 + sb), (item >> 1) & 1, p.err, s_abort));
            if (!ok) break;
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            uint32_t sv[32];
            at_ld32(trow + AT_TMEM_S + sb * AT_KEYS + half * 32, sv);
            asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
            asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
            __syncwarp();
            if (lane == 0) mbar_arrive(B(11 + sb), 1);             // this warp's part of S is in registers
            // the chunk needs the causal mask only where it reaches past this row's position (the last chunk or two of a row)
            const bool diag = j0 + 31 > t;
            if (!pass) {
                float cm = -INFINITY;
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    float sc = rbf(__uint_as_float(sv[j])) * 0.0625f;
                    if (diag && j0 + j > t) sc = -INFINITY;
                    sv[j] = __float_as_uint(sc);
                    cm = fmaxf(cm, sc);
                }
                if (live && cm != -INFINITY) {
                    const float n = fmaxf(m, cm), nl = n * AT_LOG2E;
                    float s0 = 0.f, s1 = 0.f;
#pragma unroll
                    for (int j = 0; j < 32; j += 2) {
                        s0 += at_exp2(fmaf(__uint_as_float(sv[j]), AT_LOG2E, -nl));
                        s1 += at_exp2(fmaf(__uint_as_float(sv[j + 1]), AT_LOG2E, -nl));
                    }
                    l = (m == -INFINITY ? 0.f : l * at_exp2((m - n) * AT_LOG2E)) + (s0 + s1);
                    m = n;
                }
            } else {
                const int pb = c & 1;
                if (c >= 2) ok = at_wait(B(15 + pb), ((c >> 1) - 1) & 1, p.err, s_abort);      // P V of two chunks back has read this tile
                ok = __all_sync(0xffffffffu, ok);
                if (!ok) break;
                // this thread's half of the P row: 4 pieces of 16 bytes (8 keys each), piece c8 at position c8 ^ (r mod 8)
                const float ml = m * AT_LOG2E, inv_l = (live && l > 0.f) ? 1.0f / l : 0.f;
#pragma unroll
                for (int c4 = 0; c4 < 4; ++c4) {
                    uint32_t w[4];
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        float pv[2];
#pragma unroll
                        for (int h2 = 0; h2 < 2; ++h2) {
                            const int jj = c4 * 8 + 2 * e + h2;
                            const float sc = rbf(__uint_as_float(sv[jj])) * 0.0625f;
                            pv[h2] = at_exp2(fmaf(sc, AT_LOG2E, -ml)) * inv_l;
                            if (diag && j0 + jj > t) pv[h2] = 0.f;
                        }
                        const __nv_bfloat162 pr = __floats2bfloat162_rn(pv[0], pv[1]);
                        w[e] = *reinterpret_cast<const uint32_t*>(&pr);
                    }
                    const int c8 = half * 4 + c4;
                    *reinterpret_cast<uint4*>(p_ptr + pb * AT_P_BYTES + r * 128 + ((c8 ^ (r & 7)) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
                }
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");      // generic-proxy writes -> visible to the MMA
                __syncwarp();
                if (lane == 0) mbar_arrive(B(13 + pb), 1);
            }
        }
        }
        // ---- output: bf16(P.V) * bf16(sigmoid(gate)); this thread's 128 of the row's 256 dimensions ----
        ok = __all_sync(0xffffffffu, at_wait(B(17), 0, p.err, s_abort) && ok && !*s_abort);
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        if (ok) {
            const bf16* gate = p.proj + (size_t)t * p.ldp + head * 2 * FA_HEAD_DIM + FA_HEAD_DIM;
            bf16* dst = p.out + (size_t)t * FA_Q_SIZE + head * FA_HEAD_DIM;
#pragma unroll 1
            for (int cb = half * 4; cb < half * 4 + 4; ++cb) {
                uint32_t ov[32];
                at_ld32(trow + (uint32_t)(cb * 32), ov);
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
                if (live) {
#pragma unroll
                    for (int j = 0; j < 32; j += 8) {
                        const uint4 gr = *reinterpret_cast<const uint4*>(gate + cb * 32 + j);
                        const uint32_t gw[4] = {gr.x, gr.y, gr.z, gr.w};
                        uint32_t o[4];
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            const __nv_bfloat162 pr = __halves2bfloat162(f2bf(rbf(__uint_as_float(ov[j + 2 * e])) * rbf(sigmoid_f(bf_lo(gw[e])))),
                                                                         f2bf(rbf(__uint_as_float(ov[j + 2 * e + 1])) * rbf(sigmoid_f(bf_hi(gw[e])))));
                            o[e] = *reinterpret_cast<const uint32_t*>(&pr);
                        }
                        *reinterpret_cast<uint4*>(dst + cb * 32 + j) = make_uint4(o[0], o[1], o[2], o[3]);
                    }
                }
            }
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 1) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(AT_TMEM_COLS) : "memory");
    }
}

size_t attention_tcgen05_scratch_bytes(int S) {
    const size_t s_pad = ((size_t)S + AT_KEYS - 1) / AT_KEYS * AT_KEYS;
    return (size_t)FA_KV_HEADS * FA_HEAD_DIM * s_pad * sizeof(bf16);
}

// q [S][2048] (normed, rotated), k_cache / v_cache: this layer's [2][max_seq][256], proj: gate source, out [S][2048];
// vt_scratch: attention_tcgen05_scratch_bytes(S) bytes, 1024-byte aligned
int attention_prefill_tcgen05(const bf16* q, const bf16* k_cache, const bf16* v_cache, const bf16* proj, int ldp, bf16* out, bf16* vt_scratch, int S,
                              int max_seq, cudaStream_t stream) {
    int* err = (int*)get_workspace();
    if (!err) return QWEN35_ERR_CUDA;
    static PerDeviceOnce attr;
    if (attr.pending()) {
        Q35_CUDA_OK(cudaFuncSetAttribute(attention_tcgen05_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)AT_SMEM));
        attr.mark();
    }
    const int s_pad = (S + AT_KEYS - 1) / AT_KEYS * AT_KEYS;
    Q35_CUDA_OK(pdl_launch(att_transpose_v_kernel, dim3(s_pad / 64, FA_HEAD_DIM / 64, FA_KV_HEADS), 256, 0, stream, v_cache, vt_scratch, S, s_pad, max_seq));
    CUtensorMap tmQ, tmK, tmVT;
    {
        const unsigned long long dq[3] = {(unsigned long long)FA_HEAD_DIM, (unsigned long long)FA_Q_HEADS, (unsigned long long)S};
        const unsigned long long sq[2] = {(unsigned long long)FA_HEAD_DIM * 2, (unsigned long long)FA_Q_SIZE * 2};
        const unsigned bq[3] = {64, FA_GQA, AT_Q};
        const unsigned long long dk[2] = {(unsigned long long)FA_HEAD_DIM, (unsigned long long)FA_KV_HEADS * max_seq};
        const unsigned long long sk[1] = {(unsigned long long)FA_HEAD_DIM * 2};
        const unsigned bk[2] = {64, AT_KEYS};
        const unsigned long long dv[2] = {(unsigned long long)s_pad, (unsigned long long)FA_KV_HEADS * FA_HEAD_DIM};
        const unsigned long long sv[1] = {(unsigned long long)s_pad * 2};
        const unsigned bv[2] = {AT_KEYS, FA_HEAD_DIM};
        if (!make_tmap_bf16(&tmQ, q, 3, dq, sq, bq) || !make_tmap_bf16(&tmK, k_cache, 2, dk, sk, bk) || !make_tmap_bf16(&tmVT, vt_scratch, 2, dv, sv, bv)) {
            set_error("prefill attention: tensor map creation failed (q %p, k %p, vT %p)", (const void*)q, (const void*)k_cache, (const void*)vt_scratch);
            return QWEN35_ERR_CUDA;
        }
    }
    AttParams p{proj, ldp, out, S, max_seq, err};
    Q35_CUDA_OK(pdl_launch(attention_tcgen05_kernel, dim3((S + AT_Q - 1) / AT_Q, FA_KV_HEADS), AT_THREADS, AT_SMEM, stream, tmQ, tmK, tmVT, p));
    g_launches.fetch_add(2);
    return QWEN35_OK;
}

}  // namespace q35
