// Prefill kernels of the Qwen3.5-0.8B hybrid network other than the tensor-core GEMMs:
// row norms, DeltaNet preparation (causal conv + SiLU + L2 norm, beta / log-decay), the chunk-64
// gated delta rule in two kernels (chunk-local triangular solve, then the scan over chunks),
// gated norm, q/k norm + RoPE + KV-cache fill, causal GQA attention and the last-token LM head.
//
// These replace pf_embed / pf_rmsnorm / pf_deltanet_prepare_qk / pf_deltanet_recurrence_tiled /
// pf_deltanet_finalize / pf_qk_norm_rope / pf_causal_attn_posblock / pf_lm_head of the reference
// (models/qwen35_0p8b/prefill.cu:118-892).  The reference runs the delta rule token by token
// (:385-544, 85 % of its prefill time); here it is the chunked (WY) form with all products in f32.
// Rounding points follow a bf16 HuggingFace model: every module output is rounded to bf16 once.
#pragma once

#include <cuda_fp16.h>
#include <cuda_fp4.h>
#include <cuda_fp8.h>

#include "common.cuh"
#include "nvfp4_act.cuh"

namespace q35 {

constexpr int DN_CHUNK = 64;

// ---- one CTA (128 threads) per token: optional embedding gather, RMSNorm(1+w) -------------------
// h_out (may be null) receives the raw row; x_out (may be null) the normalised row.  With q_packed / q_scales the normalised
// row is also packed as the NVFP4 activation operand of the GEMM that follows (a block of 16 elements is two threads; the
// grid then covers the rows up to the next multiple of 128, and the rows from S on are written as zeros).
// EARLY (decode steps: a handful of blocks in front of a GEMM): the GEMM is let in at once and loads weights beside this kernel
template <bool EARLY = false>
static __global__ void __launch_bounds__(128) pf_rmsnorm_kernel(const int* __restrict__ ids, const bf16* __restrict__ embed,
                                                         const bf16* __restrict__ h_in, const bf16* __restrict__ w,
                                                         bf16* __restrict__ h_out, bf16* __restrict__ x_out, int S,
                                                         uint8_t* __restrict__ q_packed, uint8_t* __restrict__ q_scales) {
    if (EARLY) pdl_trigger();
    pdl_wait();
    __shared__ float red[4];
    const int t = blockIdx.x, tid = threadIdx.x;
    if (t >= S) {                   // padding rows of the packed operand
        if (q_packed) {
            reinterpret_cast<uint32_t*>(q_packed + (size_t)t * (HIDDEN / 2))[tid] = 0u;
            if (!(tid & 1)) q_scales[nvfp4_scale_index(t, tid >> 1, HIDDEN)] = 0;
        }
        return;
    }
    const bf16* src = ids ? embed + (size_t)ids[t] * HIDDEN : h_in + (size_t)t * HIDDEN;
    const uint4 raw = *(reinterpret_cast<const uint4*>(src) + tid);
    if (h_out) *(reinterpret_cast<uint4*>(h_out + (size_t)t * HIDDEN) + tid) = raw;
    float x[8];
    x[0] = bf_lo(raw.x); x[1] = bf_hi(raw.x); x[2] = bf_lo(raw.y); x[3] = bf_hi(raw.y);
    x[4] = bf_lo(raw.z); x[5] = bf_hi(raw.z); x[6] = bf_lo(raw.w); x[7] = bf_hi(raw.w);
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) ss += x[i] * x[i];
    ss = warp_sum(ss);
    if ((tid & 31) == 0) red[tid >> 5] = ss;
    __syncthreads();
    const float tot = (red[0] + red[1]) + (red[2] + red[3]);
    const float r = rsqrt_ieee(tot * (1.0f / HIDDEN) + RMS_EPS);
    const uint4 wr = __ldg(reinterpret_cast<const uint4*>(w) + tid);
    const float wv[8] = {bf_lo(wr.x), bf_hi(wr.x), bf_lo(wr.y), bf_hi(wr.y), bf_lo(wr.z), bf_hi(wr.z), bf_lo(wr.w), bf_hi(wr.w)};
    uint32_t o[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const __nv_bfloat162 p = __halves2bfloat162(f2bf((x[2 * i] * r) * (1.0f + wv[2 * i])), f2bf((x[2 * i + 1] * r) * (1.0f + wv[2 * i + 1])));
        o[i] = *reinterpret_cast<const uint32_t*>(&p);
    }
    if (x_out) *(reinterpret_cast<uint4*>(x_out + (size_t)t * HIDDEN) + tid) = make_uint4(o[0], o[1], o[2], o[3]);
    if (q_packed) {
        const float a8 = nvfp4_amax8(o);
        float inv;
        const uint8_t s8 = nvfp4_act_scale(fmaxf(a8, __shfl_xor_sync(0xffffffffu, a8, 1)), inv);
        reinterpret_cast<uint32_t*>(q_packed + (size_t)t * (HIDDEN / 2))[tid] = nvfp4_pack8(o, inv);
        if (!(tid & 1)) q_scales[nvfp4_scale_index(t, tid >> 1, HIDDEN)] = s8;
    }
}

// ---- silu(gate) * up over [S, INTER] bf16 buffers, 8 values per thread: the epilogue of the fused [gate; up] GEMM as a
// kernel of its own, for callers whose tables hold gate and up as two matrices.  Same roundings: bf16(silu(g)) * u -> bf16.
static __global__ void __launch_bounds__(256) pf_silu_mul_kernel(const bf16* __restrict__ gate, const bf16* __restrict__ up, bf16* __restrict__ out, int n8) {
    pdl_wait();
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n8) return;
    const uint4 g = reinterpret_cast<const uint4*>(gate)[i], u = reinterpret_cast<const uint4*>(up)[i];
    const uint32_t gw[4] = {g.x, g.y, g.z, g.w}, uw[4] = {u.x, u.y, u.z, u.w};
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const __nv_bfloat162 pr = __halves2bfloat162(f2bf(rbf(silu_f(bf_lo(gw[j]))) * bf_lo(uw[j])), f2bf(rbf(silu_f(bf_hi(gw[j]))) * bf_hi(uw[j])));
        o[j] = *reinterpret_cast<const uint32_t*>(&pr);
    }
    reinterpret_cast<uint4*>(out)[i] = make_uint4(o[0], o[1], o[2], o[3]);
}

// the same over one [S, 2 * INTER] buffer whose rows hold [gate | up] (output of the fused NVFP4 gate/up GEMM)
static __global__ void __launch_bounds__(256) pf_silu_mul_rows_kernel(const bf16* __restrict__ gu, bf16* __restrict__ out, int S) {
    pdl_wait();
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= S * (INTER / 8)) return;
    const int t = i / (INTER / 8), c = i % (INTER / 8);
    const uint4 g = reinterpret_cast<const uint4*>(gu + (size_t)t * 2 * INTER)[c], u = reinterpret_cast<const uint4*>(gu + (size_t)t * 2 * INTER + INTER)[c];
    const uint32_t gw[4] = {g.x, g.y, g.z, g.w}, uw[4] = {u.x, u.y, u.z, u.w};
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const __nv_bfloat162 pr = __halves2bfloat162(f2bf(rbf(silu_f(bf_lo(gw[j]))) * bf_lo(uw[j])), f2bf(rbf(silu_f(bf_hi(gw[j]))) * bf_hi(uw[j])));
        o[j] = *reinterpret_cast<const uint32_t*>(&pr);
    }
    reinterpret_cast<uint4*>(out + (size_t)t * INTER)[c] = make_uint4(o[0], o[1], o[2], o[3]);
}

// arg-max over one row of bf16 logits (lowest index among equal maxima), optional f32 copy of the row; one CTA of 1024 threads
static __global__ void __launch_bounds__(1024) pf_argmax_row_kernel(const bf16* __restrict__ logits, int* __restrict__ out_token, float* __restrict__ logits_out) {
    pdl_wait();
    __shared__ float sv[32];
    __shared__ int si[32];
    const int tid = threadIdx.x;
    float best = -INFINITY;
    int best_i = 0x7fffffff;
    for (int c = tid; c < VOCAB; c += 1024) {
        const float f = bf2f(logits[c]);
        if (logits_out) logits_out[c] = f;
        if (f > best) { best = f; best_i = c; }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float v = __shfl_xor_sync(0xffffffffu, best, o); const int k = __shfl_xor_sync(0xffffffffu, best_i, o);
        if (v > best || (v == best && k < best_i)) { best = v; best_i = k; }
    }
    if ((tid & 31) == 0) { sv[tid >> 5] = best; si[tid >> 5] = best_i; }
    __syncthreads();
    if (tid < 32) {
        best = sv[tid]; best_i = si[tid];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float v = __shfl_xor_sync(0xffffffffu, best, o); const int k = __shfl_xor_sync(0xffffffffu, best_i, o);
            if (v > best || (v == best && k < best_i)) { best = v; best_i = k; }
        }
        if (tid == 0 && out_token) *out_token = best_i;
    }
}

// ---- DeltaNet preparation: one warp per (token, head), a lane takes four adjacent dimensions of q, k and v ------------
// proj: [S, ldp] bf16 rows [qkv 6144 | z 2048 | b 16 | a 16].  Writes qkv_out [S, 6144] bf16 (q, k L2-normalised
// in bf16 arithmetic, v after conv + SiLU), beta [S,16] (bf16-rounded sigmoid), g [S,16] (f32 log-decay), and the conv window
// the decode steps continue from.
constexpr int DN_PREP_WARPS = 8;
static __global__ void __launch_bounds__(32 * DN_PREP_WARPS) pf_dn_prep_kernel(const bf16* __restrict__ proj, int ldp, const bf16* __restrict__ conv_w,
                                                         const bf16* __restrict__ a_log, const bf16* __restrict__ dt_bias,
                                                         bf16* __restrict__ qkv_out, float* __restrict__ beta, float* __restrict__ g,
                                                         float* __restrict__ conv_state, int S) {
    pdl_wait();
    const int unit = blockIdx.x * DN_PREP_WARPS + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (unit >= S * DN_HEADS) return;
    const int t = unit / DN_HEADS, h = unit % DN_HEADS;
    float c[3][4];
#pragma unroll
    for (int part = 0; part < 3; ++part) {
        const int ch = part * DN_QK_SIZE + h * DN_K + 4 * lane;
        const uint4 w01 = __ldg(reinterpret_cast<const uint4*>(conv_w + (size_t)ch * 4));         // taps of channels ch, ch + 1
        const uint4 w23 = __ldg(reinterpret_cast<const uint4*>(conv_w + (size_t)ch * 4) + 1);     // ch + 2, ch + 3
        const uint32_t wr[8] = {w01.x, w01.y, w01.z, w01.w, w23.x, w23.y, w23.z, w23.w};
        uint2 xr[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int tt = t - 3 + j;
            xr[j] = (tt >= 0) ? *reinterpret_cast<const uint2*>(proj + (size_t)tt * ldp + ch) : make_uint2(0u, 0u);
        }
        if (t == S - 1) {
            // the last token's four taps are the conv window after the prompt: the last four inputs per channel, zero-padded
            // on the left, newest last (f32 [channel][4])
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                float4 w;
                w.x = (e & 1) ? bf_hi(e < 2 ? xr[0].x : xr[0].y) : bf_lo(e < 2 ? xr[0].x : xr[0].y);
                w.y = (e & 1) ? bf_hi(e < 2 ? xr[1].x : xr[1].y) : bf_lo(e < 2 ? xr[1].x : xr[1].y);
                w.z = (e & 1) ? bf_hi(e < 2 ? xr[2].x : xr[2].y) : bf_lo(e < 2 ? xr[2].x : xr[2].y);
                w.w = (e & 1) ? bf_hi(e < 2 ? xr[3].x : xr[3].y) : bf_lo(e < 2 ? xr[3].x : xr[3].y);
                reinterpret_cast<float4*>(conv_state)[ch + e] = w;
            }
        }
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const float w4[4] = {bf_lo(wr[2 * e]), bf_hi(wr[2 * e]), bf_lo(wr[2 * e + 1]), bf_hi(wr[2 * e + 1])};
            float acc = 0.f;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const uint32_t pair = (e < 2) ? xr[j].x : xr[j].y;
                const float xv = (e & 1) ? bf_hi(pair) : bf_lo(pair);
                acc = (j == 0) ? w4[j] * xv : fmaf(w4[j], xv, acc);
            }
            c[part][e] = rbf(silu_f(rbf(acc)));
        }
    }
    // L2 norm of q and k in bf16 arithmetic: squares rounded, f32 sum rounded once, + eps, rsqrt, scale.
    // torch's vectorised CPU rsqrt rounds once; its scalar tail (the last S*16 mod 32 elements, i.e. the last
    // token when S is odd) rounds sqrt to bf16 first.  The oracle is that CPU path, so both are mirrored.
    const bool scalar_tail = (S & 1) && (t == S - 1);
#pragma unroll
    for (int part = 0; part < 2; ++part) {
        float tot = warp_sum(((rbf(c[part][0] * c[part][0]) + rbf(c[part][1] * c[part][1])) + rbf(c[part][2] * c[part][2])) + rbf(c[part][3] * c[part][3]));
        tot = rbf(rbf(tot) + 1e-6f);
        const float inv = scalar_tail ? rbf(1.0f / rbf(sqrtf(tot))) : rbf(rsqrt_ieee(tot));
#pragma unroll
        for (int e = 0; e < 4; ++e) c[part][e] = rbf(c[part][e] * inv);
    }
    bf16* dst = qkv_out + (size_t)t * DN_CONV_CH + h * DN_K + 4 * lane;
#pragma unroll
    for (int part = 0; part < 3; ++part) {
        const __nv_bfloat162 lo = __floats2bfloat162_rn(c[part][0], c[part][1]), hi = __floats2bfloat162_rn(c[part][2], c[part][3]);
        *reinterpret_cast<uint2*>(dst + part * DN_QK_SIZE) = make_uint2(*reinterpret_cast<const uint32_t*>(&lo), *reinterpret_cast<const uint32_t*>(&hi));
    }
    if (lane == 0) {
        const float bb = bf2f(proj[(size_t)t * ldp + DN_CONV_CH + DN_V_SIZE + h]);
        const float aa = bf2f(proj[(size_t)t * ldp + DN_CONV_CH + DN_V_SIZE + DN_HEADS + h]);
        beta[t * DN_HEADS + h] = rbf(sigmoid_f(bb));
        const float x = aa + bf2f(dt_bias[h]);
        const float sp = (x > 20.f) ? x : log1pf(expf(x));
        g[t * DN_HEADS + h] = -expf(bf2f(a_log[h])) * sp;
    }
}

// ---- TF32 tensor-core helpers (legacy mma.sync path, m16n8k8) --------------------------------------------------------
// The chunk kernels multiply f32 matrices whose results feed a recurrent f32 state, so plain TF32 (10 mantissa bits) is
// not enough.  Each operand is split x = hi + lo with hi = tf32(x), lo = tf32(x - hi), and a product is taken as
// a_lo b_hi + a_hi b_lo + a_hi b_hi with f32 accumulation ("3xTF32"): about 21 bits per operand, f32 sums.
// Fragment layout of mma.m16n8k8 (g = lane / 4, t = lane % 4):  A (16x8, row):  a0 (g, t)  a1 (g+8, t)  a2 (g, t+4)  a3 (g+8, t+4);
// B (8x8, k x n):  b0 (t, g)  b1 (t+4, g);   C (16x8):  c0 (g, 2t)  c1 (g, 2t+1)  c2 (g+8, 2t)  c3 (g+8, 2t+1).
// f32 -> tf32, round to nearest with ties away from zero: what cvt.rna.tf32.f32 returns for finite values, written as an
// add and a mask on the bit pattern (sign-magnitude, so adding half a last place to the magnitude rounds it).  The
// conversion instruction runs at a fraction of the integer rate and bounded these kernels.
__device__ __forceinline__ uint32_t tf32_of(float x) { return (__float_as_uint(x) + 0x1000u) & 0xffffe000u; }
__device__ __forceinline__ void tf32_split(float x, uint32_t& hi, uint32_t& lo) {
    hi = tf32_of(x);
    lo = tf32_of(x - __uint_as_float(hi));
}
__device__ __forceinline__ void mma_tf32(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile("mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                 : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
// One accumulator per term: three independent dependency chains instead of one three times as long (the kernels below are
// bound by the latency of back-to-back mma on one accumulator, not by issue slots); the terms are summed small to large.
__device__ __forceinline__ void mma_3xtf32_terms(float (&c)[3][4], const uint32_t (&ah)[4], const uint32_t (&al)[4], uint32_t bh0, uint32_t bh1,
                                                 uint32_t bl0, uint32_t bl1) {
    mma_tf32(c[0], al, bh0, bh1);
    mma_tf32(c[1], ah, bl0, bl1);
    mma_tf32(c[2], ah, bh0, bh1);
}
__device__ __forceinline__ float sum_terms(const float (&c)[3][4], int r) { return (c[0][r] + c[1][r]) + c[2][r]; }
// A fragment of a row-major f32 matrix in shared memory (rows m0.., columns k0..), split into hi / lo
__device__ __forceinline__ void load_a_split(const float* A, int ld, int m0, int k0, uint32_t (&ah)[4], uint32_t (&al)[4]) {
    const int g = (threadIdx.x & 31) >> 2, t = threadIdx.x & 3;
    tf32_split(A[(m0 + g) * ld + k0 + t], ah[0], al[0]);
    tf32_split(A[(m0 + g + 8) * ld + k0 + t], ah[1], al[1]);
    tf32_split(A[(m0 + g) * ld + k0 + t + 4], ah[2], al[2]);
    tf32_split(A[(m0 + g + 8) * ld + k0 + t + 4], ah[3], al[3]);
}
// ---- chunk-local part of the gated delta rule: one CTA (16 warps) per (chunk, head) --------------
// Per chunk of 64 tokens (zero padded): gc = cumsum(g); T = (I + tril((k beta) k^T * decay, -1))^-1 (a unit lower triangular
// solve); vprime = T (v beta); aqk = tril(q k^T * decay).  f32 throughout; the three matrix products (k k^T, q k^T, T v) run
// on the tensor cores with q, k, v as exact tf32 operands (they are bf16 values) and only T split hi + lo; the triangular
// solve runs on the CUDA cores in 16 x 16 blocks.
// The record the scan kernel reads.  Every one of its 8 value slices of a head reads the shared part of the record, so the
// record is kept small: q and k stay the bf16 values they are, T and aqk keep only the 16-row tiles' columns up to the
// diagonal block, and the product T (k beta exp(gc)) of the chunk-64 formulation is not formed at all (the scan multiplies
// k S first, a 64 x 16 matrix, and T after).  q and k are stored as the scan's tcgen05 operands, in the K-major 128-byte-swizzle
// layout the MMA reads (rows of 128 bytes, the 16-byte unit u of row r at position u ^ (r & 7)): qk = the 128 x 128 left operand
// [k rows; q rows] of (k S, q S) as two blocks of 64 dims, kt = k^T (128 dims x 64 tokens), the left operand of the state
// update.  Each group of arrays that lands together is contiguous, so it moves with one bulk copy; pad columns are never read.
constexpr int SCAN_VW = 16;                 // value columns per scan CTA
// T and aqk: row tile m (16 rows) holds columns 0 .. 16 (m + 1) - 1 at pitch 16 (m + 1) + 8 floats (8 or 24 mod 32: the
// 64-bit fragment loads of a half warp, rows g = 0..3, fall in different banks)
__host__ __device__ constexpr int tri_pitch(int m) { return 16 * (m + 1) + 8; }
__host__ __device__ constexpr int tri_off(int m) { return 128 * m * (m + 2); }
constexpr int SCAN_TRI = tri_off(4);        // 3072 floats
struct ChunkScratch {          // one record per (head, chunk); every array starts on a 16-byte boundary
    float vprime[DN_V / SCAN_VW][DN_CHUNK][SCAN_VW];     // by 16-column slice: a scan CTA copies its own
    bf16 qk[2][2 * DN_CHUNK][64];      // copy 1: [block of 64 dims][k tokens, then q tokens][dim], swizzled
    bf16 kt[DN_K][DN_CHUNK];           //         [dim][token], swizzled
    float tmat[SCAN_TRI];              // copy 2: T, aqk and the four vectors
    float aqk[SCAN_TRI];
    float wsc[DN_CHUNK];               // beta_i exp(gc_i):       scales row i of k S
    float dq[DN_CHUNK];                // exp(gc_i) / sqrt(128):  scales row i of q S
    float kdec[DN_CHUNK];              // exp(gc_last - gc_i):    scales row i of v_new for the state update
    float eg_last[4];                  // [0] = exp(gc_last)
};
static_assert(sizeof(ChunkScratch) % 16 == 0, "records must keep 16-byte alignment");
constexpr uint32_t SCAN_QK_BYTES = 2 * 2 * DN_CHUNK * 64 * 2, SCAN_KT_BYTES = DN_K * DN_CHUNK * 2,
                   SCAN_TA_BYTES = (2 * SCAN_TRI + 3 * DN_CHUNK + 4) * 4, SCAN_VP_BYTES = DN_CHUNK * SCAN_VW * 4;
static_assert(offsetof(ChunkScratch, kt) == offsetof(ChunkScratch, qk) + SCAN_QK_BYTES &&
              offsetof(ChunkScratch, eg_last) + 16 == offsetof(ChunkScratch, tmat) + SCAN_TA_BYTES, "the copies assume this layout");
// byte offset of the 16-byte unit holding elements col .. col + 7 of row `row` in a swizzled block of 128-byte rows
__host__ __device__ constexpr uint32_t sw128_off(int row, int col) { return (uint32_t)row * 128u + ((uint32_t)((col >> 3) ^ (row & 7)) << 4); }

constexpr int CL_THREADS = 512;
constexpr float CL_QSCALE = 0.08838834764831845f;        // 1 / sqrt(128)
constexpr int CL_LD = DN_K + 4;                          // q, k: A operands (row-major) and, for k, the transposed B operand: bank = 4 g + t
constexpr int CL_LDB = DN_K + 8;                         // v: B operand [token][dim]: bank = 8 t + g
constexpr int CL_LDA = DN_CHUNK + 4;                     // T: A operand of the last product
// q and v share one region (v replaces q once q k^T is done): 107 KB, so that two CTAs fit an SM and the phases of one
// (loads, tensor-core products, the triangular solve on a few warps) run under those of the other
constexpr int CHUNK_LOCAL_SMEM = (DN_CHUNK * CL_LD + DN_CHUNK * CL_LDB + 2 * DN_CHUNK * CL_LDA + 3 * 256 + 3 * DN_CHUNK) * 4;

static __global__ void __launch_bounds__(CL_THREADS, 2) pf_dn_chunk_local_kernel(const bf16* __restrict__ qkv, const float* __restrict__ beta,
                                                                       const float* __restrict__ g, ChunkScratch* __restrict__ scratch,
                                                                       int S, int nchunks) {
    pdl_wait();
    extern __shared__ __align__(16) float sm[];
    float* sq = sm;                                  // [64][CL_LD]   q, until q k^T is done; then
    float* sv = sm;                                  // [64][CL_LDB]  v (held in registers meanwhile)
    float* sk = sm + DN_CHUNK * CL_LDB;              // [64][CL_LD]   k
    float* sa = sk + DN_CHUNK * CL_LD;               // [64][CL_LDA]  N = -(k beta) k^T * decay, strictly lower
    float* sx = sa + DN_CHUNK * CL_LDA;              // [64][CL_LDA]  T = (I - N)^-1
    float* sw = sx + DN_CHUNK * CL_LDA;              // [3][16][16]   block products of the inversion
    float* sb = sw + 3 * 256;
    float* sg = sb + DN_CHUNK;      // cumulative log-decay
    float* se = sg + DN_CHUNK;      // exp(gc)
    const int c = blockIdx.x, h = blockIdx.y, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int gq = lane >> 2, t4 = lane & 3;
    const int t0 = c * DN_CHUNK;
    ChunkScratch& out = scratch[(size_t)h * nchunks + c];

    if (tid < DN_CHUNK) {
        const int t = t0 + tid;
        sb[tid] = (t < S) ? beta[t * DN_HEADS + h] : 0.f;
        sg[tid] = (t < S) ? g[t * DN_HEADS + h] : 0.f;
    }
    static_assert(DN_CHUNK * (DN_K / 8) == 2 * CL_THREADS, "two 16-byte pieces of each of q, k, v per thread");
    uint4 vreg[2];
#pragma unroll
    for (int it = 0; it < 2; ++it) {                                          // eight dimensions (16 bytes of bf16) per step
        const int e = tid + it * CL_THREADS;
        const int i = e >> 4, d = (e & 15) * 8, t = t0 + i;
        uint4 qr = make_uint4(0, 0, 0, 0), kr = qr, vr = qr;
        if (t < S) {
            const bf16* row = qkv + (size_t)t * DN_CONV_CH + h * DN_K + d;
            qr = *reinterpret_cast<const uint4*>(row);
            kr = *reinterpret_cast<const uint4*>(row + DN_QK_SIZE);
            vr = *reinterpret_cast<const uint4*>(row + 2 * DN_QK_SIZE);
        }
        // q and k stay the bf16 values they are (8 significant bits: exact as tf32 operands); the 1 / sqrt(128) of q is applied to
        // the products below.  The scan reads the same bf16 rows (zero for padding tokens).
        {
            unsigned char* blk = reinterpret_cast<unsigned char*>(&out.qk[d >> 6][0][0]);
            *reinterpret_cast<uint4*>(blk + sw128_off(i, d & 63)) = kr;
            *reinterpret_cast<uint4*>(blk + sw128_off(DN_CHUNK + i, d & 63)) = qr;
        }
        *reinterpret_cast<float4*>(sq + i * CL_LD + d) = make_float4(bf_lo(qr.x), bf_hi(qr.x), bf_lo(qr.y), bf_hi(qr.y));
        *reinterpret_cast<float4*>(sq + i * CL_LD + d + 4) = make_float4(bf_lo(qr.z), bf_hi(qr.z), bf_lo(qr.w), bf_hi(qr.w));
        *reinterpret_cast<float4*>(sk + i * CL_LD + d) = make_float4(bf_lo(kr.x), bf_hi(kr.x), bf_lo(kr.y), bf_hi(kr.y));
        *reinterpret_cast<float4*>(sk + i * CL_LD + d + 4) = make_float4(bf_lo(kr.z), bf_hi(kr.z), bf_lo(kr.w), bf_hi(kr.w));
        vreg[it] = vr;
    }
    __syncthreads();
    if (tid == 0) {                 // sequential cumsum, as torch.cumsum does
        float acc = 0.f;
        for (int i = 0; i < DN_CHUNK; ++i) { acc += sg[i]; sg[i] = acc; }
    }
    __syncthreads();
    // k^T for the scan's state update: eight tokens of one dim are one 16-byte unit
    for (int e = tid; e < DN_K * (DN_CHUNK / 8); e += CL_THREADS) {
        const int d = e & (DN_K - 1), ju = e >> 7;
        uint32_t w[4];
#pragma unroll
        for (int jj = 0; jj < 4; ++jj)
            w[jj] = (__float_as_uint(sk[(ju * 8 + 2 * jj) * CL_LD + d]) >> 16) | (__float_as_uint(sk[(ju * 8 + 2 * jj + 1) * CL_LD + d]) & 0xffff0000u);
        *reinterpret_cast<uint4*>(reinterpret_cast<unsigned char*>(&out.kt[0][0]) + sw128_off(d, ju * 8)) = make_uint4(w[0], w[1], w[2], w[3]);
    }
    if (tid < DN_CHUNK) {            // the per-token factors of the scan
        const float e = expf(sg[tid]);
        se[tid] = e;
        out.wsc[tid] = sb[tid] * e;
        out.dq[tid] = CL_QSCALE * e;
        out.kdec[tid] = expf(sg[DN_CHUNK - 1] - sg[tid]);
        if (tid == 0) out.eg_last[0] = expf(sg[DN_CHUNK - 1]);
    }
    __syncthreads();
    // ---- k k^T and q k^T (64 x 64 x 128): only the tiles on and below the diagonal.  A = rows of k (warps 0-7) or q (8-15),
    // B = k^T.  Eight warps share the 20 lower-triangular 16 x 8 ... tiles of one product: (row tile, first column tile, count)
    {
        const int u = warp & 7;
        const int mt = (u < 3) ? 3 : (u < 5) ? 2 : (u < 7) ? 1 : 0;
        const int nt0 = (u == 1 || u == 4) ? 3 : (u == 2) ? 6 : (u == 6) ? 2 : 0;
        const int ntn = (u == 2 || u >= 5) ? 2 : 3;
        const bool is_q = warp >= 8;
        const float* A = is_q ? sq : sk;
        // Both operands are bf16 values, exact in tf32: one MMA per tile and k-step, no hi / lo split (the f32 products of the
        // chunk-64 formulation, summed on the tensor cores).  Two halves of the k range on separate accumulators.
        float acc2[2][3][4];
#pragma unroll
        for (int e = 0; e < 24; ++e) acc2[e / 12][(e >> 2) % 3][e & 3] = 0.f;
#pragma unroll 2
        for (int k0 = 0; k0 < DN_K / 2; k0 += 8) {
#pragma unroll
            for (int hf = 0; hf < 2; ++hf) {
                const int kk = k0 + hf * (DN_K / 2);
                const float* ar = A + (mt * 16 + gq) * CL_LD + kk + t4;
                const uint32_t af[4] = {__float_as_uint(ar[0]), __float_as_uint(ar[8 * CL_LD]), __float_as_uint(ar[4]), __float_as_uint(ar[8 * CL_LD + 4])};
#pragma unroll
                for (int n = 0; n < 3; ++n)
                    if (n < ntn) {
                        const float* br = sk + ((nt0 + n) * 8 + gq) * CL_LD + kk + t4;        // B(k, n) = k[token n][dim k]
                        mma_tf32(acc2[hf][n], af, __float_as_uint(br[0]), __float_as_uint(br[4]));
                    }
            }
        }
        float acc[3][4];
#pragma unroll
        for (int n = 0; n < 3; ++n)
#pragma unroll
            for (int r = 0; r < 4; ++r) acc[n][r] = acc2[0][n][r] + acc2[1][n][r];
        // A[i][j] = -(beta_i k_i . k_j) * exp(gc_i - gc_j) for j < i, else 0;   aqk[i][j] = (q_i . k_j) * exp(gc_i - gc_j) for j <= i
#pragma unroll
        for (int n = 0; n < 3; ++n)
            if (n < ntn)
#pragma unroll
                for (int r = 0; r < 4; ++r) {
                    const int i = mt * 16 + gq + 8 * (r >> 1), j = (nt0 + n) * 8 + 2 * t4 + (r & 1);
                    const float dec = (j <= i) ? expf(sg[i] - sg[j]) : 0.f;
                    if (is_q) out.aqk[tri_off(mt) + (i & 15) * tri_pitch(mt) + j] = (j <= i) ? (acc[n][r] * CL_QSCALE) * dec : 0.f;
                    else sa[i * CL_LDA + j] = (j < i) ? -((acc[n][r] * sb[i]) * dec) : 0.f;
                }
        // the tiles above the diagonal blocks were not computed: A is zero there (the forward substitution reads column
        // entries above the diagonal and relies on their being zero); aqk does not store them
        for (int e = tid; e < DN_CHUNK * DN_CHUNK; e += CL_THREADS) {
            const int i = e >> 6, j = e & 63;
            if ((j >> 4) > (i >> 4)) sa[i * CL_LDA + j] = 0.f;
        }
    }
    __syncthreads();
    // q is no longer read: v takes its place (read by the last product, several barriers from here)
#pragma unroll
    for (int it = 0; it < 2; ++it) {
        const int e = tid + it * CL_THREADS;
        const int i = e >> 4, d = (e & 15) * 8;
        const uint4 vr = vreg[it];
        *reinterpret_cast<float4*>(sv + i * CL_LDB + d) = make_float4(bf_lo(vr.x), bf_hi(vr.x), bf_lo(vr.y), bf_hi(vr.y));
        *reinterpret_cast<float4*>(sv + i * CL_LDB + d + 4) = make_float4(bf_lo(vr.z), bf_hi(vr.z), bf_lo(vr.w), bf_hi(vr.w));
    }
    // T = (I - N)^-1 with N = sa (strictly lower triangular), in 16 x 16 blocks.
    //   diagonal blocks: forward substitution inside the block (T_ij = N_ij + sum_{j < k < i} N_ik T_kj), one warp per block,
    //   one lane per column, so its 15 steps need no barrier at all;
    //   blocks below: T_ij = T_ii * sum_{k = j}^{i-1} N_ik T_kj, one block diagonal at a time (three levels), each level two small
    //   products on the CUDA cores.  The same triangular solve as the row-by-row loop of the chunk-64 formulation, summed in
    //   block order.
    if (warp < 4 && lane < 16) {
        // lane j solves column j of the block on its own: x_i = N_ij + sum_{j < k < i} N_ik x_k, the x_k in registers, the rows
        // of N read as broadcasts; no step waits for another lane
        const float* blk = sa + (warp * 16) * CL_LDA + warp * 16;
        float x[16];
        x[0] = 0.f;
#pragma unroll
        for (int i = 1; i < 16; ++i) {
            float nrow[16];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const float4 v = *reinterpret_cast<const float4*>(blk + i * CL_LDA + 4 * q);
                nrow[4 * q] = v.x; nrow[4 * q + 1] = v.y; nrow[4 * q + 2] = v.z; nrow[4 * q + 3] = v.w;
            }
            float a0 = 0.f, a1 = 0.f;
#pragma unroll
            for (int k = 1; k < i; ++k) {
                if (k & 1) a0 = fmaf(nrow[k], x[k], a0);
                else a1 = fmaf(nrow[k], x[k], a1);
            }
            float nij = 0.f;
#pragma unroll
            for (int k = 0; k < 16; ++k) nij = (k == lane) ? nrow[k] : nij;
            x[i] = (lane < i) ? nij + (a0 + a1) : 0.f;
        }
        // the finished block, with its unit diagonal and zero upper triangle, into T
#pragma unroll
        for (int i = 0; i < 16; ++i)
            sx[(warp * 16 + i) * CL_LDA + warp * 16 + lane] = (lane < i) ? x[i] : (lane == i ? 1.0f : 0.f);
    }
    __syncthreads();
    for (int d = 1; d < 4; ++d) {
        const int nblk = 4 - d;
        // W_b = sum_{k = j}^{i-1} N_ik T_kj for the blocks (i, j) = (b + d, b)
        for (int e = tid; e < nblk * 256; e += CL_THREADS) {
            const int b = e >> 8, r = (e >> 4) & 15, cc = e & 15;
            const float* nrow = sa + ((b + d) * 16 + r) * CL_LDA + b * 16;       // N[i-row][columns of blocks j .. i-1]
            const float* tcol = sx + (b * 16) * CL_LDA + b * 16 + cc;             // T[rows of blocks j .. i-1][column]
            float a0 = 0.f, a1 = 0.f;
#pragma unroll 4
            for (int k = 0; k < 16 * d; k += 2) {
                a0 = fmaf(nrow[k], tcol[k * CL_LDA], a0);
                a1 = fmaf(nrow[k + 1], tcol[(k + 1) * CL_LDA], a1);
            }
            sw[e] = a0 + a1;
        }
        __syncthreads();
        // T_ij = T_ii W_b (T_ii lower triangular with unit diagonal)
        for (int e = tid; e < nblk * 256; e += CL_THREADS) {
            const int b = e >> 8, r = (e >> 4) & 15, cc = e & 15;
            const float* trow = sx + ((b + d) * 16 + r) * CL_LDA + (b + d) * 16;
            const float* wc = sw + b * 256 + cc;
            float a0 = 0.f, a1 = 0.f;
            for (int k = 0; k + 2 <= r; k += 2) {
                a0 = fmaf(trow[k], wc[k * 16], a0);
                a1 = fmaf(trow[k + 1], wc[(k + 1) * 16], a1);
            }
            if (r & 1) a0 = fmaf(trow[r - 1], wc[(r - 1) * 16], a0);
            sx[((b + d) * 16 + r) * CL_LDA + b * 16 + cc] = wc[r * 16] + (a0 + a1);
        }
        __syncthreads();
    }
    // ---- vprime = T (v beta): 64 x 128 x 64 with T lower triangular.  beta_j belongs to the summation index j, so it goes into
    // the left operand: T diag(beta) times the rows of v.  v is bf16 values, exact as a tf32 operand, so only the left operand
    // is split: two MMAs per tile and k-step instead of three.  T itself goes to the scan, tile rows up to the diagonal block.
    for (int e = tid; e < DN_CHUNK * DN_CHUNK; e += CL_THREADS) {
        const int i = e >> 6, j = e & 63, m = i >> 4;
        const bool in = (j >> 4) <= m;
        const float tij = in ? sx[i * CL_LDA + j] : 0.f;
        sa[i * CL_LDA + j] = tij * sb[j];                  // N is no longer needed: its buffer holds T diag(beta)
        if (in) out.tmat[tri_off(m) + (i & 15) * tri_pitch(m) + j] = tij;
    }
    __syncthreads();
    // A warp takes an eighth of the 128 columns and two row tiles whose k ranges add up to the same length: (0, 3) or (1, 2).
    {
        const int nq = warp & 7;
        const bool outer = warp < 8;
#pragma unroll
        for (int pass = 0; pass < 2; ++pass) {
            const int mt = outer ? (pass ? 3 : 0) : (pass ? 2 : 1);
            float acc2[2][2][4];
#pragma unroll
            for (int n = 0; n < 2; ++n)
#pragma unroll
                for (int r = 0; r < 8; ++r) acc2[n][r >> 2][r & 3] = 0.f;
            for (int k0 = 0; k0 < 16 * (mt + 1); k0 += 8) {
                uint32_t ah[4], al[4];
                load_a_split(sa, CL_LDA, mt * 16, k0, ah, al);
#pragma unroll
                for (int n = 0; n < 2; ++n) {
                    const float* br = sv + (k0 + t4) * CL_LDB + nq * 16 + n * 8 + gq;       // B(k, n) = v[token k][dim n]
                    const uint32_t b0 = __float_as_uint(br[0]), b1 = __float_as_uint(br[4 * CL_LDB]);
                    mma_tf32(acc2[n][0], al, b0, b1);
                    mma_tf32(acc2[n][1], ah, b0, b1);
                }
            }
#pragma unroll
            for (int n = 0; n < 2; ++n)
#pragma unroll
                for (int hr = 0; hr < 2; ++hr) {
                    const int i = mt * 16 + gq + 8 * hr, d = nq * 16 + n * 8 + 2 * t4;
                    *reinterpret_cast<float2*>(&out.vprime[d / SCAN_VW][i][d % SCAN_VW]) =
                        make_float2(acc2[n][0][2 * hr] + acc2[n][1][2 * hr], acc2[n][0][2 * hr + 1] + acc2[n][1][2 * hr + 1]);
                }
        }
    }
}

// ---- scan over chunks: one CTA (8 compute warps + a copy / MMA-issue warp) per (head, 16-wide slice of the value dimension) ----
// Sequential over the chunks of a head; with S the state slice [128 k][16 v], per chunk
//   W = w (k S),  v_new = vprime - T W,  out = d (q S) + aqk v_new,  S <- S exp(gc_last) + k^T (e v_new)
// (w_i = beta_i exp(gc_i), d_i = exp(gc_i) / sqrt(128), e_i = exp(gc_last - gc_i); T W equals the chunk-64 formulation's
// (T (k beta exp(gc))) S with the products taken in the other order).  Every product has the accuracy of f32:
//   P1  [k; q] S (128 x 128 x 16) and P3 k^T (e v_new) (128 x 64 x 16) on the 5th-generation tensor cores: tcgen05.mma
//       kind::f16 with the bf16 rows of q and k as the left operand, exact as they are, and the f32 right operand split
//       into three bf16 pieces (24 significant bits).  The pieces sit side by side as 48 columns of ONE right operand, so a
//       product is 8 (P1) or 4 (P3) instructions instead of three times as many (a 16-column instruction takes as long
//       to issue as a 48-column one); the three partial tiles are added when they are read back from tensor memory;
//   P1b T W and P2 aqk v_new (64 x 64 x 16, lower triangular, both operands f32) as 3xTF32 mma.sync tiles, the eight warps a
//       4 x 2 grid of (16-token row tile, 8-column tile), zero k-steps skipped.
// The state slice lives in registers from chunk to chunk, one row (key dim) of 8 columns per thread, as it comes out of
// tensor memory; shared memory holds its three pieces as the right operand of the next chunk's P1.  One lane of the ninth
// warp brings each chunk's operands in with three bulk copies (completion counted on an mbarrier) into one of two stages, a
// chunk ahead of the compute warps, and issues both tcgen05 products, each as soon as the compute warps have announced its
// right operand on an mbarrier (state pieces -> P1, e v_new pieces -> P3).  P2 of a chunk is not on the path to the next
// state: it runs under the next chunk's P1 (v_new and d (q S) are kept by chunk parity), and the chunk's stage is released
// after it.  Row tiles of the last chunk that hold only padding are skipped.  Every wait is bounded and sets the status word.
constexpr int SCAN_CONS = 256;              // compute threads
constexpr int SCAN_THREADS = SCAN_CONS + 32;
constexpr int SCAN_LDB = SCAN_VW + 4;       // W, v_new (hi and lo), d (q S): rows 2 t, 2 t + 1 of a k-step: bank = 8 t + g
constexpr int SCAN_NSTAGE = 2;
constexpr uint32_t SCAN_STAGE_BYTES = SCAN_QK_BYTES + SCAN_KT_BYTES + SCAN_TA_BYTES + SCAN_VP_BYTES;
constexpr uint32_t SCAN_STAGE_PITCH = (SCAN_STAGE_BYTES + 1023u) & ~1023u;       // the swizzled blocks start on 1024-byte boundaries
constexpr uint32_t SCAN_SP_BYTES = 2 * 3 * SCAN_VW * 128;       // state pieces:   [block of 64 dims][piece][value column][dim]
constexpr uint32_t SCAN_VK_BYTES = 3 * SCAN_VW * 128;           // e v_new pieces: [piece][value column][token]
constexpr int SCAN_NB = 3 * SCAN_VW;        // columns of the right operands: the three pieces side by side
constexpr int CHUNK_SCAN_SMEM = 1024 + SCAN_NSTAGE * SCAN_STAGE_PITCH + SCAN_SP_BYTES + SCAN_VK_BYTES + 8 * DN_CHUNK * SCAN_LDB * 4 + 64;
static_assert(CHUNK_SCAN_SMEM <= 227 * 1024, "the scan's operands must fit one CTA's shared memory");
constexpr uint32_t SCAN_TMEM_COLS = 128;    // two 128 x 48 f32 accumulators (allocations are powers of two)
constexpr uint32_t SCAN_D2_COL = 64;        // first column of the second accumulator
// instruction descriptor: D f32, A / B bf16, both K-major, N = 48 at [17,23) in units of 8, M = 128 at [24,29) in units of 16
constexpr uint32_t SCAN_IDESC = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(SCAN_NB >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
constexpr unsigned SCAN_WAIT_LIMIT = 1u << 26;      // a bounded wait: a copy or an MMA that never completes ends the loop instead of hanging

// (once the status word is set -- by this wait, by another thread's or by an earlier kernel -- every later wait gives up within
// a thousand polls, so a failed pass ends quickly)
__device__ __forceinline__ void scan_wait(uint32_t bar, uint32_t parity, int* err) {
    unsigned it = 0;
    while (!mbar_try_wait(bar, parity)) {
        ++it;
        if (it >= SCAN_WAIT_LIMIT) { atomicCAS(err, 0, (int)ERR_BARRIER_TIMEOUT); return; }
        if ((it & 1023u) == 0 && *reinterpret_cast<volatile int*>(err) != 0) return;
    }
}
__device__ __forceinline__ void scan_cons_sync() { asm volatile("bar.sync 1, %0;" ::"n"(SCAN_CONS) : "memory"); }
// shared-memory matrix descriptor, K-major operand, 128-byte swizzle: start address >> 4 | SBO = 1024 B between 8-row groups |
// version 1 | layout 2
__device__ __forceinline__ uint64_t scan_smem_desc(uint32_t smem_addr) {
    return (uint64_t)((smem_addr & 0x3FFFFu) >> 4) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) | ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
__device__ __forceinline__ void scan_umma(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(SCAN_IDESC), "r"(accumulate) : "memory");
}
__device__ __forceinline__ void scan_umma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
// this warp's 32 rows x 8 columns of an accumulator, one row per lane: the sum of the three partial tiles (16 columns apart),
// small to large
__device__ __forceinline__ void scan_tmem_ld8(uint32_t taddr, float (&v)[8]) {
    uint32_t r[3][8];
#pragma unroll
    for (int pc = 0; pc < 3; ++pc)
        asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                     : "=r"(r[pc][0]), "=r"(r[pc][1]), "=r"(r[pc][2]), "=r"(r[pc][3]), "=r"(r[pc][4]), "=r"(r[pc][5]), "=r"(r[pc][6]), "=r"(r[pc][7])
                     : "r"(taddr + (uint32_t)(pc * SCAN_VW)) : "memory");
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = (__uint_as_float(r[2][j]) + __uint_as_float(r[1][j])) + __uint_as_float(r[0][j]);
}
// x = p0 + p1 + p2 up to 2^-24 |x|, each piece a bf16 value (returned as its 16 bits)
__device__ __forceinline__ void bf16_split3(float x, unsigned short (&p)[3]) {
    const bf16 a = __float2bfloat16_rn(x);
    const float r1 = x - __bfloat162float(a);
    const bf16 b = __float2bfloat16_rn(r1);
    const bf16 c = __float2bfloat16_rn(r1 - __bfloat162float(b));
    p[0] = __bfloat16_as_ushort(a); p[1] = __bfloat16_as_ushort(b); p[2] = __bfloat16_as_ushort(c);
}
// (volatile keeps these stores in order with the fences and barriers, which are volatile too; no memory clobber, so that
// the loads around them are not serialised)
__device__ __forceinline__ void st_shared_u16(uint32_t addr, unsigned short v) { asm volatile("st.shared.u16 [%0], %1;" ::"r"(addr), "h"(v)); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
// 16 x 8 (x 16 (mt + 1)) product of a row tile of a packed lower-triangular matrix (T or aqk) with a split B operand; within a
// k-step of 8 the mma's k index t stands for column 2 t and t + 4 for column 2 t + 1, so a float2 is one fragment pair
__device__ __forceinline__ void scan_tri_product(float (&a3)[3][4], const float* tile, int pitch, int klen, const uint32_t* bh, const uint32_t* bl,
                                                 int col, int g, int t4) {
    const float* r0 = tile + g * pitch + 2 * t4;
    const float* r1 = r0 + 8 * pitch;
    for (int j0 = 0; j0 < klen; j0 += 8) {
        const float2 x0 = *reinterpret_cast<const float2*>(r0 + j0), x1 = *reinterpret_cast<const float2*>(r1 + j0);
        uint32_t ah[4], al[4];
        tf32_split(x0.x, ah[0], al[0]);
        tf32_split(x1.x, ah[1], al[1]);
        tf32_split(x0.y, ah[2], al[2]);
        tf32_split(x1.y, ah[3], al[3]);
        const int bi0 = (j0 + 2 * t4) * SCAN_LDB + col, bi1 = bi0 + SCAN_LDB;
        mma_3xtf32_terms(a3, ah, al, bh[bi0], bh[bi1], bl[bi0], bl[bi1]);
    }
}

static __global__ void __launch_bounds__(SCAN_THREADS) pf_dn_chunk_scan_kernel(const ChunkScratch* __restrict__ scratch, bf16* __restrict__ core_out,
                                                                        float* __restrict__ state_out, int S, int nchunks, int* __restrict__ err) {
    pdl_wait();
    extern __shared__ unsigned char scan_raw[];
    const uint32_t raw_a = smem_u32(scan_raw), base_a = (raw_a + 1023u) & ~1023u;
    unsigned char* sm0 = scan_raw + (base_a - raw_a);
    const uint32_t sp_a = base_a + SCAN_NSTAGE * SCAN_STAGE_PITCH;      // state pieces
    const uint32_t vk_a = sp_a + SCAN_SP_BYTES;                         // e v_new pieces
    uint32_t* swh = reinterpret_cast<uint32_t*>(sm0 + SCAN_NSTAGE * SCAN_STAGE_PITCH + SCAN_SP_BYTES + SCAN_VK_BYTES);      // [64][SCAN_LDB] W, hi
    uint32_t* swl = swh + DN_CHUNK * SCAN_LDB;                          //                 W, lo
    uint32_t* vnh0 = swl + DN_CHUNK * SCAN_LDB;                         // [2][64][SCAN_LDB] v_new, hi   (these three by chunk parity:
    uint32_t* vnl0 = vnh0 + 2 * DN_CHUNK * SCAN_LDB;                    //                    v_new, lo    P2 of a chunk runs during
    float* sit0 = reinterpret_cast<float*>(vnl0 + 2 * DN_CHUNK * SCAN_LDB);   // [2][64][SCAN_LDB] d (q S)   the next chunk's P1)
    u64* bars = reinterpret_cast<u64*>(sit0 + 2 * DN_CHUNK * SCAN_LDB);  // full[2], empty[2], P1 done, P3 done, state ready, e v_new ready
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * SCAN_NSTAGE + 4);
    const int h = blockIdx.x, vs = blockIdx.y, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, t4 = lane & 3;
    const int v0 = vs * SCAN_VW;
    const uint32_t full0 = smem_u32(bars), empty0 = full0 + 8 * SCAN_NSTAGE, p1bar = empty0 + 8 * SCAN_NSTAGE, p3bar = p1bar + 8;
    const uint32_t sready = p3bar + 8, vkready = sready + 8;
    if (tid == 0) {
        for (int i = 0; i < SCAN_NSTAGE; ++i) {
            mbar_init(full0 + 8 * i, 1);
            mbar_init(empty0 + 8 * i, SCAN_CONS / 32);       // one arrival per compute warp
        }
        mbar_init(p1bar, 1);
        mbar_init(p3bar, 1);
        mbar_init(sready, SCAN_CONS / 32);
        mbar_init(vkready, SCAN_CONS / 32);
        mbar_fence_init();
    }
    for (uint32_t e = tid; e < SCAN_SP_BYTES / 4; e += SCAN_THREADS) reinterpret_cast<uint32_t*>(sm0 + SCAN_NSTAGE * SCAN_STAGE_PITCH)[e] = 0u;   // state = 0
    fence_async_smem();
    if (warp == SCAN_CONS / 32) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)), "r"(SCAN_TMEM_COLS) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == SCAN_CONS / 32) {
        // ---- copy and MMA warp (one lane issues both): copies run a chunk ahead; an MMA goes out as soon as its right operand
        // is announced complete, so no compute warp waits on the issue itself ----
        if (lane == 0) {
            auto issue_copy = [&](int c) {
                const ChunkScratch& in = scratch[(size_t)h * nchunks + c];
                const int sg = c % SCAN_NSTAGE, use = c / SCAN_NSTAGE;
                if (use > 0) scan_wait(empty0 + 8 * sg, (use - 1) & 1, err);
                const uint32_t full = full0 + 8 * sg, dst = base_a + sg * SCAN_STAGE_PITCH;
                mbar_arrive_expect_tx(full, SCAN_STAGE_BYTES);
                bulk_load_1d(dst, &in.qk[0][0][0], SCAN_QK_BYTES + SCAN_KT_BYTES, full);
                bulk_load_1d(dst + SCAN_QK_BYTES + SCAN_KT_BYTES, &in.tmat[0], SCAN_TA_BYTES, full);
                bulk_load_1d(dst + SCAN_QK_BYTES + SCAN_KT_BYTES + SCAN_TA_BYTES, &in.vprime[vs][0][0], SCAN_VP_BYTES, full);
            };
            issue_copy(0);
            for (int c = 0; c < nchunks; ++c) {
                const int sg = c % SCAN_NSTAGE;
                const uint32_t qk_a = base_a + sg * SCAN_STAGE_PITCH, kt_a = qk_a + SCAN_QK_BYTES;
                scan_wait(full0 + 8 * sg, (c / SCAN_NSTAGE) & 1, err);             // this chunk's operands have landed (long ago)
                if (c > 0) scan_wait(sready, (c - 1) & 1, err);                    // the state's pieces after chunk c - 1
                tc_fence_after();
                // ---- P1: [k; q] [S0 | S1 | S2] ----
#pragma unroll
                for (int kb = 0; kb < 2; ++kb) {
                    const uint64_t adesc = scan_smem_desc(qk_a + kb * (SCAN_QK_BYTES / 2)), bdesc = scan_smem_desc(sp_a + kb * (SCAN_SP_BYTES / 2));
#pragma unroll
                    for (int ks = 0; ks < 4; ++ks) scan_umma(tmem_base, adesc + 2 * ks, bdesc + 2 * ks, (kb > 0 || ks > 0) ? 1u : 0u);
                }
                scan_umma_commit(p1bar);
                if (c + 1 < nchunks) issue_copy(c + 1);        // its stage is released by P2 of chunk c - 1, which runs now
                // ---- P3: k^T [e v_new 0 | 1 | 2] over the k-steps of 16 tokens that hold tokens ----
                scan_wait(vkready, c & 1, err);
                tc_fence_after();
                const int nks = (min(DN_CHUNK, S - c * DN_CHUNK) + 15) >> 4;
                const uint64_t adesc = scan_smem_desc(kt_a), bdesc = scan_smem_desc(vk_a);
#pragma unroll
                for (int ks = 0; ks < 4; ++ks)
                    if (ks < nks) scan_umma(tmem_base + SCAN_D2_COL, adesc + 2 * ks, bdesc + 2 * ks, ks > 0 ? 1u : 0u);
                scan_umma_commit(p3bar);
            }
        }
        __syncwarp();
    } else {
        // this thread's row of the state slice: key dim 32 (warp & 3) + lane, value columns 8 (warp >> 2) .. + 7, f32
        float st8[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) st8[j] = 0.f;
        const int q4 = warp & 3, ch = warp >> 2, drow = 32 * q4 + lane;
        const uint32_t tm_d1 = tmem_base + ((uint32_t)(32 * q4) << 16) + (uint32_t)(8 * ch), tm_d2 = tm_d1 + SCAN_D2_COL;
        // where this row's pieces go in the right operand of P1: [dims / 64][piece][value column][dim % 64], swizzled
        const uint32_t sp_row = sp_a + (uint32_t)(drow >> 6) * (SCAN_SP_BYTES / 2) + (uint32_t)ch * 1024u + (uint32_t)(drow & 7) * 2u;
        // the warp's tile of the 64 x 16 mma.sync products: the two warps of a scheduler (warp and warp + 4) take row tiles mt and
        // 3 - mt, whose triangular products add up to the same length
        const int nt = warp >> 2, mt = nt ? 3 - (warp & 3) : (warp & 3), m0 = mt * 16, col = nt * 8 + g;

        // ---- P2 of chunk cp: out = d (q S) + aqk v_new.  Not on the path to the next chunk's state, so it runs while the tensor
        // cores work on the next chunk's P1 (after the last chunk: on its own); the chunk's stage is released after it ----
        auto p2 = [&](int cp) {
            const int tp = cp * DN_CHUNK, sgp = cp % SCAN_NSTAGE;
            if (mt * 16 < S - tp) {
                const float* sAp = reinterpret_cast<const float*>(sm0 + sgp * SCAN_STAGE_PITCH + SCAN_QK_BYTES + SCAN_KT_BYTES) + SCAN_TRI;
                const uint32_t* vh = vnh0 + (cp & 1) * DN_CHUNK * SCAN_LDB;
                const uint32_t* vl = vnl0 + (cp & 1) * DN_CHUNK * SCAN_LDB;
                const float* si = sit0 + (cp & 1) * DN_CHUNK * SCAN_LDB;
                float a3[3][4];
#pragma unroll
                for (int i = 0; i < 12; ++i) a3[i >> 2][i & 3] = 0.f;
                scan_tri_product(a3, sAp + tri_off(mt), tri_pitch(mt), 16 * (mt + 1), vh, vl, col, g, t4);
#pragma unroll
                for (int hr = 0; hr < 2; ++hr) {
                    const int row = m0 + g + 8 * hr, tok = tp + row;
                    if (tok < S) {
                        const float2 it = *reinterpret_cast<const float2*>(si + row * SCAN_LDB + nt * 8 + 2 * t4);
                        bf16* dst = core_out + (size_t)tok * DN_V_SIZE + h * DN_V + v0 + nt * 8 + 2 * t4;
                        *reinterpret_cast<__nv_bfloat162*>(dst) =
                            __halves2bfloat162(f2bf(it.x + sum_terms(a3, 2 * hr)), f2bf(it.y + sum_terms(a3, 2 * hr + 1)));
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(empty0 + 8 * sgp, 1);               // this warp is done with the stage
        };

        for (int c = 0; c < nchunks; ++c) {
            const int t0 = c * DN_CHUNK;
            const int sg = c % SCAN_NSTAGE;
            const float* sT = reinterpret_cast<const float*>(sm0 + sg * SCAN_STAGE_PITCH + SCAN_QK_BYTES + SCAN_KT_BYTES);
            const float* sA = sT + SCAN_TRI;
            const float* swsc = sA + SCAN_TRI;
            const float* sdq = swsc + DN_CHUNK;
            const float* skd = sdq + DN_CHUNK;
            const float* seg = skd + DN_CHUNK;
            const float* svp = seg + 4;
            const int valid = min(DN_CHUNK, S - t0);
            const bool live = mt * 16 < valid;                    // this row tile holds at least one token
            uint32_t* vnh = vnh0 + (c & 1) * DN_CHUNK * SCAN_LDB;
            uint32_t* vnl = vnl0 + (c & 1) * DN_CHUNK * SCAN_LDB;
            float* sit = sit0 + (c & 1) * DN_CHUNK * SCAN_LDB;
            scan_wait(full0 + 8 * sg, (c / SCAN_NSTAGE) & 1, err);            // this chunk's operands have landed
            const float dec = seg[0];
            if (c > 0) p2(c - 1);
            scan_wait(p1bar, c & 1, err);
            __syncwarp();
            tc_fence_after();
            {
                float v[8];
                scan_tmem_ld8(tm_d1, v);
                if (q4 < 2) {            // rows of k S: W = w (k S), split, as the B operand of P1b
                    const float w = swsc[drow];
                    uint32_t hi[8], lo[8];
#pragma unroll
                    for (int j = 0; j < 8; ++j) tf32_split(v[j] * w, hi[j], lo[j]);
                    uint4* dh = reinterpret_cast<uint4*>(swh + drow * SCAN_LDB + 8 * ch);
                    uint4* dl = reinterpret_cast<uint4*>(swl + drow * SCAN_LDB + 8 * ch);
                    dh[0] = make_uint4(hi[0], hi[1], hi[2], hi[3]); dh[1] = make_uint4(hi[4], hi[5], hi[6], hi[7]);
                    dl[0] = make_uint4(lo[0], lo[1], lo[2], lo[3]); dl[1] = make_uint4(lo[4], lo[5], lo[6], lo[7]);
                } else {                 // rows of q S: d (q S), for P2
                    const float d = sdq[drow - DN_CHUNK];
                    float4* di = reinterpret_cast<float4*>(sit + (drow - DN_CHUNK) * SCAN_LDB + 8 * ch);
                    di[0] = make_float4(v[0] * d, v[1] * d, v[2] * d, v[3] * d);
                    di[1] = make_float4(v[4] * d, v[5] * d, v[6] * d, v[7] * d);
                }
            }
            tc_fence_before();
            scan_cons_sync();                                              // W and d (q S) complete
            // ---- P1b: v_new = vprime - T W, stored split for P2 and, with row i scaled by e_i, in three bf16 pieces for P3 ----
            if (live) {
                float a3[3][4];
#pragma unroll
                for (int i = 0; i < 12; ++i) a3[i >> 2][i & 3] = 0.f;
                scan_tri_product(a3, sT + tri_off(mt), tri_pitch(mt), 16 * (mt + 1), swh, swl, col, g, t4);
                float vpv[4], kdv[2];
#pragma unroll
                for (int r = 0; r < 4; ++r) vpv[r] = svp[(m0 + g + 8 * (r >> 1)) * SCAN_VW + nt * 8 + 2 * t4 + (r & 1)];
                kdv[0] = skd[m0 + g];
                kdv[1] = skd[m0 + g + 8];
#pragma unroll
                for (int r = 0; r < 4; ++r) {
                    const int row = m0 + g + 8 * (r >> 1), cv = nt * 8 + 2 * t4 + (r & 1);
                    const float vn = vpv[r] - sum_terms(a3, r);
                    uint32_t hi, lo;
                    tf32_split(vn, hi, lo);
                    vnh[row * SCAN_LDB + cv] = hi;
                    vnl[row * SCAN_LDB + cv] = lo;
                    unsigned short pcs[3];
                    bf16_split3(vn * kdv[r >> 1], pcs);
                    const uint32_t a = vk_a + (uint32_t)nt * 1024u + (uint32_t)(cv & 7) * 128u + ((uint32_t)((row >> 3) ^ (cv & 7)) << 4) + (uint32_t)(row & 7) * 2u;
                    st_shared_u16(a, pcs[0]);
                    st_shared_u16(a + 2048, pcs[1]);
                    st_shared_u16(a + 4096, pcs[2]);
                }
            }
            fence_async_smem();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(vkready, 1);                        // this warp's part of the right operand of P3 is written
            scan_cons_sync();                                              // v_new complete (P2 reads it in the next iteration)
            // ---- the new state: S exp(gc_last) + P3, in registers and in pieces for the next chunk's P1 ----
            scan_wait(p3bar, c & 1, err);
            __syncwarp();
            tc_fence_after();
            {
                float v[8];
                scan_tmem_ld8(tm_d2, v);
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    st8[j] = fmaf(st8[j], dec, v[j]);
                    unsigned short pcs[3];
                    bf16_split3(st8[j], pcs);
                    const uint32_t a = sp_row + (uint32_t)j * 128u + ((uint32_t)(((drow & 63) >> 3) ^ j) << 4);
                    st_shared_u16(a, pcs[0]);
                    st_shared_u16(a + 2048, pcs[1]);
                    st_shared_u16(a + 4096, pcs[2]);
                }
            }
            fence_async_smem();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(sready, 1);                         // this warp's rows of the next P1's right operand are written
        }
        p2(nchunks - 1);
        // final state in the reference layout [head][v][k], from the f32 registers
#pragma unroll
        for (int j = 0; j < 8; ++j) state_out[((size_t)h * DN_V + v0 + 8 * ch + j) * DN_K + drow] = st8[j];
    }
    tc_fence_before();
    __syncthreads();
    if (warp == SCAN_CONS / 32) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(SCAN_TMEM_COLS) : "memory");
    }
}

// ---- gated RMSNorm of the DeltaNet output: half a warp per (token, head) -----------------------------
template <bool EARLY = false>
static __global__ void __launch_bounds__(256) pf_gated_norm_kernel(const bf16* __restrict__ core, const bf16* __restrict__ proj, int ldp,
                                                            const bf16* __restrict__ norm_w, bf16* __restrict__ out, int S) {
    if (EARLY) pdl_trigger();
    pdl_wait();
    // half a warp per (token, head): 16 lanes x 8 values, 16-byte loads and stores
    const int lane = threadIdx.x & 31, l16 = lane & 15;
    const int gw = (blockIdx.x * 8 + (threadIdx.x >> 5)) * 2 + (lane >> 4);
    const bool live = gw < S * DN_HEADS;
    const int t = live ? gw / DN_HEADS : 0, h = live ? gw % DN_HEADS : 0;
    uint4 orw = make_uint4(0, 0, 0, 0), zrw = orw;
    if (live) {
        orw = *(reinterpret_cast<const uint4*>(core + (size_t)t * DN_V_SIZE + h * DN_V) + l16);
        zrw = *(reinterpret_cast<const uint4*>(proj + (size_t)t * ldp + DN_CONV_CH + h * DN_V) + l16);
    }
    const uint4 nrw = __ldg(reinterpret_cast<const uint4*>(norm_w) + l16);
    const uint32_t ow[4] = {orw.x, orw.y, orw.z, orw.w}, zw[4] = {zrw.x, zrw.y, zrw.z, zrw.w}, nwd[4] = {nrw.x, nrw.y, nrw.z, nrw.w};
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) ss += bf_lo(ow[i]) * bf_lo(ow[i]) + bf_hi(ow[i]) * bf_hi(ow[i]);
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);          // within the half warp
    const float r = rsqrt_ieee(ss * (1.0f / DN_V) + RMS_EPS);
    uint32_t res[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float u0 = rbf(bf_lo(nwd[i]) * rbf(bf_lo(ow[i]) * r)) * silu_f(bf_lo(zw[i]));
        const float u1 = rbf(bf_hi(nwd[i]) * rbf(bf_hi(ow[i]) * r)) * silu_f(bf_hi(zw[i]));
        const __nv_bfloat162 pr = __halves2bfloat162(f2bf(u0), f2bf(u1));
        res[i] = *reinterpret_cast<const uint32_t*>(&pr);
    }
    if (live) *(reinterpret_cast<uint4*>(out + (size_t)t * DN_V_SIZE + h * DN_V) + l16) = make_uint4(res[0], res[1], res[2], res[3]);
}

// ---- attention preparation: one warp per (token, head slot); slots 0-7 query heads, 8-9 key heads, 10-11 value heads
// proj rows: [per head q(256) | gate(256)] x 8, k 512, v 512.  q -> q_out [S, 2048]; k, v -> cache rows [kv_head][t][256].
struct RopeTable { float f[FA_ROT / 2]; };

static __global__ void __launch_bounds__(256) pf_qk_norm_rope_kernel(const bf16* __restrict__ proj, int ldp, const bf16* __restrict__ qn_w,
                                                              const bf16* __restrict__ kn_w, const RopeTable inv_freq,
                                                              bf16* __restrict__ q_out, bf16* __restrict__ k_cache, bf16* __restrict__ v_cache,
                                                              int S, int max_seq) {
    pdl_wait();
    const int gw = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (gw >= S * 12) return;
    const int t = gw / 12, slot = gw % 12;
    if (slot >= 10) {
        const int kvh = slot - 10;
        const uint4 v = *(reinterpret_cast<const uint4*>(proj + (size_t)t * ldp + FA_QPROJ + FA_KV_SIZE + kvh * FA_HEAD_DIM) + lane);
        *(reinterpret_cast<uint4*>(v_cache + ((size_t)kvh * max_seq + t) * FA_HEAD_DIM) + lane) = v;
        return;
    }
    const bool isq = slot < 8;
    const bf16* src = proj + (size_t)t * ldp + (isq ? slot * 2 * FA_HEAD_DIM : FA_QPROJ + (slot - 8) * FA_HEAD_DIM);
    const bf16* nw = isq ? qn_w : kn_w;
    float xv[8], ss = 0.f;       // xv[i] = element lane + 32 i
#pragma unroll
    for (int i = 0; i < 8; ++i) { xv[i] = bf2f(src[lane + 32 * i]); ss += xv[i] * xv[i]; }
    const float r = rsqrt_ieee(warp_sum(ss) * (1.0f / FA_HEAD_DIM) + RMS_EPS);
#pragma unroll
    for (int i = 0; i < 8; ++i) xv[i] = rbf((xv[i] * r) * (1.0f + bf2f(nw[lane + 32 * i])));
    const float ang = (float)t * inv_freq.f[lane];
    const float cs = rbf(cosf(ang)), sn = rbf(sinf(ang));
    const float x1 = xv[0], x2 = xv[1];
    xv[0] = rbf(rbf(x1 * cs) + rbf(-x2 * sn));
    xv[1] = rbf(rbf(x2 * cs) + rbf(x1 * sn));
    bf16* dst = isq ? q_out + (size_t)t * FA_Q_SIZE + slot * FA_HEAD_DIM : k_cache + ((size_t)(slot - 8) * max_seq + t) * FA_HEAD_DIM;
#pragma unroll
    for (int i = 0; i < 8; ++i) dst[lane + 32 * i] = f2bf(xv[i]);
}

constexpr int ATT_PF_MAX_S = 4096;      // longest prompt the prefill entry points accept

// ---- last-token LM head: GEMV over the vocabulary + arg-max (lowest index among equal bf16 maxima) -----
static __global__ void __launch_bounds__(256) pf_lm_head_kernel(const bf16* __restrict__ x, const bf16* __restrict__ lm, float* __restrict__ bmv,
                                                         int* __restrict__ bmi, float* __restrict__ logits_out) {
    pdl_wait();
    __shared__ float sv[8];
    __shared__ int si[8];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float xr[32];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const uint4 v = *(reinterpret_cast<const uint4*>(x) + j * 32 + lane);
        xr[8 * j + 0] = bf_lo(v.x); xr[8 * j + 1] = bf_hi(v.x); xr[8 * j + 2] = bf_lo(v.y); xr[8 * j + 3] = bf_hi(v.y);
        xr[8 * j + 4] = bf_lo(v.z); xr[8 * j + 5] = bf_hi(v.z); xr[8 * j + 6] = bf_lo(v.w); xr[8 * j + 7] = bf_hi(v.w);
    }
    const int r0 = part_begin(VOCAB, blockIdx.x, gridDim.x), r1 = part_begin(VOCAB, blockIdx.x + 1, gridDim.x);
    float best = -INFINITY;
    int best_i = 0x7fffffff;
    for (int r = r0 + warp; r < r1; r += 8) {
        const uint4* wr = reinterpret_cast<const uint4*>(lm + (size_t)r * HIDDEN) + lane;
        float a = 0.f;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const uint4 q = ld_stream(wr + j * 32);
            a = fmaf(bf_lo(q.x), xr[8 * j + 0], a); a = fmaf(bf_hi(q.x), xr[8 * j + 1], a);
            a = fmaf(bf_lo(q.y), xr[8 * j + 2], a); a = fmaf(bf_hi(q.y), xr[8 * j + 3], a);
            a = fmaf(bf_lo(q.z), xr[8 * j + 4], a); a = fmaf(bf_hi(q.z), xr[8 * j + 5], a);
            a = fmaf(bf_lo(q.w), xr[8 * j + 6], a); a = fmaf(bf_hi(q.w), xr[8 * j + 7], a);
        }
        const float v = rbf(warp_sum(a));
        if (lane == 0 && logits_out) logits_out[r] = v;
        if (v > best) { best = v; best_i = r; }
    }
    if (lane == 0) { sv[warp] = best; si[warp] = best_i; }
    __syncthreads();
    if (threadIdx.x == 0) {
        float bv = sv[0]; int bi = si[0];
        for (int w = 1; w < 8; ++w) if (sv[w] > bv || (sv[w] == bv && si[w] < bi)) { bv = sv[w]; bi = si[w]; }
        bmv[blockIdx.x] = bv; bmi[blockIdx.x] = bi;
    }
}

static __global__ void pf_lm_reduce_kernel(const float* __restrict__ bmv, const int* __restrict__ bmi, int n, int* __restrict__ out_token) {
    pdl_wait();
    float bv = -INFINITY; int bi = 0x7fffffff;
    for (int i = threadIdx.x; i < n; i += 32) {
        const float v = bmv[i]; const int k = bmi[i];
        if (v > bv || (v == bv && k < bi)) { bv = v; bi = k; }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float v = __shfl_xor_sync(0xffffffffu, bv, o); const int k = __shfl_xor_sync(0xffffffffu, bi, o);
        if (v > bv || (v == bv && k < bi)) { bv = v; bi = k; }
    }
    if (threadIdx.x == 0) *out_token = bi;
}

}  // namespace q35
