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

namespace q35 {

constexpr int DN_CHUNK = 64;

// ---- one CTA (128 threads) per token: optional embedding gather, RMSNorm(1+w) -------------------
// h_out (may be null) receives the raw row; x_out the normalised row.
static __global__ void __launch_bounds__(128) pf_rmsnorm_kernel(const int* __restrict__ ids, const bf16* __restrict__ embed,
                                                         const bf16* __restrict__ h_in, const bf16* __restrict__ w,
                                                         bf16* __restrict__ h_out, bf16* __restrict__ x_out, int S) {
    pdl_wait();
    __shared__ float red[4];
    const int t = blockIdx.x, tid = threadIdx.x;
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
    *(reinterpret_cast<uint4*>(x_out + (size_t)t * HIDDEN) + tid) = make_uint4(o[0], o[1], o[2], o[3]);
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
// A = M^T with M holding values that are exact in tf32 (bf16 inputs): the bits go to the mma as they are
__device__ __forceinline__ void load_at_exact(const float* M, int ld, int m0, int k0, uint32_t (&a)[4]) {
    const int g = (threadIdx.x & 31) >> 2, t = threadIdx.x & 3;
    a[0] = __float_as_uint(M[(k0 + t) * ld + m0 + g]);
    a[1] = __float_as_uint(M[(k0 + t) * ld + m0 + g + 8]);
    a[2] = __float_as_uint(M[(k0 + t + 4) * ld + m0 + g]);
    a[3] = __float_as_uint(M[(k0 + t + 4) * ld + m0 + g + 8]);
}

// ---- chunk-local part of the gated delta rule: one CTA (16 warps) per (chunk, head) --------------
// Per chunk of 64 tokens (zero padded): gc = cumsum(g); T = (I + tril((k beta) k^T * decay, -1))^-1 (a unit lower triangular
// solve); vprime = T (v beta); kcd = T (k beta exp(gc)); aqk = tril(q k^T * decay).  f32 throughout; the four matrix products
// (k k^T, q k^T, T v, T k) run on the tensor cores with q, k, v as exact tf32 operands (they are bf16 values) and only T split
// hi + lo; the triangular solve runs on the CUDA cores in 16 x 16 blocks.
// The record the scan kernel reads.  Its arrays have the row pitches of the scan's shared-memory operands (padded against
// bank conflicts) and vprime is stored by 16-column slice, so that each operand of a scan CTA is ONE contiguous block
// and moves with a single bulk copy; the pad columns are never read by an mma.
constexpr int SCAN_VW = 16;                 // value columns per scan CTA
constexpr int SCAN_LDA = DN_K + 4;          // kcd, qs: row-major A operands, bank = 4 g + t
constexpr int SCAN_LDT = DN_K + 8;          // ks: read as its transpose, bank = 8 t + g
constexpr int SCAN_LDQ = DN_CHUNK + 4;      // aqk
struct ChunkScratch {          // one record per (head, chunk), floats; every array starts on a 16-byte boundary
    float vprime[DN_V / SCAN_VW][DN_CHUNK][SCAN_VW];
    float kcd[DN_CHUNK][SCAN_LDA];
    float qs[DN_CHUNK][SCAN_LDA];      // q / sqrt(128) * exp(gc_i): the scan's left operand of q S
    float ks[DN_CHUNK][SCAN_LDT];      // k as read (bf16 values):   the scan's left operand of the state update, exact in tf32
    float aqk[DN_CHUNK][SCAN_LDQ];
    float kdec[DN_CHUNK];              // exp(gc_last - gc_i): the scan scales row i of v_new by it for the state update (follows aqk: one copy)
    float eg_last[4];              // [0] = exp(gc_last)
};
static_assert(sizeof(ChunkScratch) % 16 == 0, "records must keep 16-byte alignment");

constexpr int CL_THREADS = 512;
constexpr float CL_QSCALE = 0.08838834764831845f;        // 1 / sqrt(128)
constexpr int CL_LD = DN_K + 4;                          // q, k: A operands (row-major) and, for k, the transposed B operand: bank = 4 g + t
constexpr int CL_LDB = DN_K + 8;                         // v beta, k beta exp(gc): B operands [token][dim]: bank = 8 t + g
constexpr int CL_LDA = DN_CHUNK + 4;                     // T: A operand of the last two products
constexpr int CHUNK_LOCAL_SMEM = (2 * DN_CHUNK * CL_LD + 2 * DN_CHUNK * CL_LDB + 2 * DN_CHUNK * CL_LDA + 3 * 256 + 3 * DN_CHUNK) * 4;

static __global__ void __launch_bounds__(CL_THREADS) pf_dn_chunk_local_kernel(const bf16* __restrict__ qkv, const float* __restrict__ beta,
                                                                       const float* __restrict__ g, ChunkScratch* __restrict__ scratch,
                                                                       int S, int nchunks) {
    pdl_wait();
    extern __shared__ __align__(16) float sm[];
    float* sq = sm;                                  // [64][CL_LD]   q / sqrt(128)
    float* sk = sq + DN_CHUNK * CL_LD;               // [64][CL_LD]   k
    float* sv = sk + DN_CHUNK * CL_LD;               // [64][CL_LDB]  v
    float* skb = sv + DN_CHUNK * CL_LDB;             // [64][CL_LDB]  k again, in the B-operand pitch
    float* sa = skb + DN_CHUNK * CL_LDB;             // [64][CL_LDA]  N = -(k beta) k^T * decay, strictly lower
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
    for (int e = tid; e < DN_CHUNK * (DN_K / 8); e += CL_THREADS) {          // eight dimensions (16 bytes of bf16) per step
        const int i = e >> 4, d = (e & 15) * 8, t = t0 + i;
        uint4 qr = make_uint4(0, 0, 0, 0), kr = qr, vr = qr;
        if (t < S) {
            const bf16* row = qkv + (size_t)t * DN_CONV_CH + h * DN_K + d;
            qr = *reinterpret_cast<const uint4*>(row);
            kr = *reinterpret_cast<const uint4*>(row + DN_QK_SIZE);
            vr = *reinterpret_cast<const uint4*>(row + 2 * DN_QK_SIZE);
        }
        // q and k stay the bf16 values they are (8 significant bits: exact as tf32 operands); the 1 / sqrt(128) of q is applied to
        // the products below
        *reinterpret_cast<float4*>(sq + i * CL_LD + d) = make_float4(bf_lo(qr.x), bf_hi(qr.x), bf_lo(qr.y), bf_hi(qr.y));
        *reinterpret_cast<float4*>(sq + i * CL_LD + d + 4) = make_float4(bf_lo(qr.z), bf_hi(qr.z), bf_lo(qr.w), bf_hi(qr.w));
        *reinterpret_cast<float4*>(sk + i * CL_LD + d) = make_float4(bf_lo(kr.x), bf_hi(kr.x), bf_lo(kr.y), bf_hi(kr.y));
        *reinterpret_cast<float4*>(sk + i * CL_LD + d + 4) = make_float4(bf_lo(kr.z), bf_hi(kr.z), bf_lo(kr.w), bf_hi(kr.w));
        *reinterpret_cast<float4*>(sv + i * CL_LDB + d) = make_float4(bf_lo(vr.x), bf_hi(vr.x), bf_lo(vr.y), bf_hi(vr.y));
        *reinterpret_cast<float4*>(sv + i * CL_LDB + d + 4) = make_float4(bf_lo(vr.z), bf_hi(vr.z), bf_lo(vr.w), bf_hi(vr.w));
    }
    __syncthreads();
    if (tid == 0) {                 // sequential cumsum, as torch.cumsum does
        float acc = 0.f;
        for (int i = 0; i < DN_CHUNK; ++i) { acc += sg[i]; sg[i] = acc; }
    }
    __syncthreads();
    if (tid < DN_CHUNK) { se[tid] = expf(sg[tid]); out.kdec[tid] = expf(sg[DN_CHUNK - 1] - sg[tid]); }
    __syncthreads();
    {   // operands of the scan that depend on this chunk only; a copy of k in the B-operand pitch for the products below
        const float g_last = sg[DN_CHUNK - 1];
        for (int e = tid; e < DN_CHUNK * (DN_K / 4); e += CL_THREADS) {
            const int i = e >> 5, d = (e & 31) * 4;
            const float4 kv = *reinterpret_cast<const float4*>(sk + i * CL_LD + d), qv = *reinterpret_cast<const float4*>(sq + i * CL_LD + d);
            const float ei = se[i];
            *reinterpret_cast<float4*>(&out.qs[i][d]) = make_float4((qv.x * CL_QSCALE) * ei, (qv.y * CL_QSCALE) * ei, (qv.z * CL_QSCALE) * ei, (qv.w * CL_QSCALE) * ei);
            *reinterpret_cast<float4*>(&out.ks[i][d]) = kv;
            *reinterpret_cast<float4*>(skb + i * CL_LDB + d) = kv;
        }
        if (tid == 0) out.eg_last[0] = expf(g_last);
    }
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
                    if (is_q) out.aqk[i][j] = (j <= i) ? (acc[n][r] * CL_QSCALE) * dec : 0.f;
                    else sa[i * CL_LDA + j] = (j < i) ? -((acc[n][r] * sb[i]) * dec) : 0.f;
                }
        // the tiles above the diagonal blocks were not computed: aqk and A are zero there (the forward substitution reads
        // column entries above the diagonal and relies on their being zero)
        for (int e = tid; e < DN_CHUNK * DN_CHUNK; e += CL_THREADS) {
            const int i = e >> 6, j = e & 63;
            if ((j >> 4) > (i >> 4)) { out.aqk[i][j] = 0.f; sa[i * CL_LDA + j] = 0.f; }
        }
    }
    __syncthreads();
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
    // ---- vprime = T (v beta) (warps 0-7), kcd = T (k beta exp(gc)) (warps 8-15): 64 x 128 x 64 with T lower triangular.
    // beta_j and beta_j exp(gc_j) belong to the summation index j, so they go into the left operand: T diag(beta) times the
    // rows of v, T diag(beta exp(gc)) times the rows of k.  v and k are bf16 values, exact as tf32 operands, so only the
    // left operand is split: two MMAs per tile and k-step instead of three, and no split of the right operand.
    for (int e = tid; e < DN_CHUNK * DN_CHUNK; e += CL_THREADS) {
        const int i = e >> 6, j = e & 63;
        const float tij = (j >> 4) <= (i >> 4) ? sx[i * CL_LDA + j] : 0.f;
        sa[i * CL_LDA + j] = tij * sb[j];                  // N is no longer needed: its buffer holds T diag(beta)
        sx[i * CL_LDA + j] = tij * (sb[j] * se[j]);
    }
    __syncthreads();
    // A warp takes a quarter of the 128 columns and two row tiles whose k ranges add up to the same length: (0, 3) or (1, 2).
    {
        const int u = warp & 7, nq = u & 3;
        const bool to_vp = warp < 8;
        const float* Bm = to_vp ? sv : skb;
        const float* Am = to_vp ? sa : sx;
#pragma unroll
        for (int pass = 0; pass < 2; ++pass) {
            const int mt = (u < 4) ? (pass ? 3 : 0) : (pass ? 2 : 1);
            float acc2[4][2][4];
#pragma unroll
            for (int n = 0; n < 4; ++n)
#pragma unroll
                for (int r = 0; r < 8; ++r) acc2[n][r >> 2][r & 3] = 0.f;
            for (int k0 = 0; k0 < 16 * (mt + 1); k0 += 8) {
                uint32_t ah[4], al[4];
                load_a_split(Am, CL_LDA, mt * 16, k0, ah, al);
#pragma unroll
                for (int n = 0; n < 4; ++n) {
                    const float* br = Bm + (k0 + t4) * CL_LDB + nq * 32 + n * 8 + gq;       // B(k, n) = Bm[token k][dim n]
                    const uint32_t b0 = __float_as_uint(br[0]), b1 = __float_as_uint(br[4 * CL_LDB]);
                    mma_tf32(acc2[n][0], al, b0, b1);
                    mma_tf32(acc2[n][1], ah, b0, b1);
                }
            }
#pragma unroll
            for (int n = 0; n < 4; ++n)
#pragma unroll
                for (int hr = 0; hr < 2; ++hr)
                {
                    const int i = mt * 16 + gq + 8 * hr, d = nq * 32 + n * 8 + 2 * t4;
                    float* dst = to_vp ? &out.vprime[d / SCAN_VW][i][d % SCAN_VW] : &out.kcd[i][d];
                    *reinterpret_cast<float2*>(dst) = make_float2(acc2[n][0][2 * hr] + acc2[n][1][2 * hr], acc2[n][0][2 * hr + 1] + acc2[n][1][2 * hr + 1]);
                }
        }
    }
}

// ---- scan over chunks: one CTA (8 warps) per (head, 16-wide slice of the value dimension) --------
// Sequential over the chunks of a head; per chunk  v_new = vprime - kcd S,  out = qs S + aqk v_new,
// S <- S exp(gc_last) + k^T (e v_new)  (S = state slice [128 k][16 v]).  All four products run on the tensor cores as
// 3xTF32 mma.sync tiles (two terms where the left operand is exact):
//   P1  warps 0-3: VP = kcd S, warps 4-7: IT = qs S      (64 x 128 x 16, one 16-row tile and both 8-column tiles per warp)
//   P2  warps 4-7: out = IT + aqk v_new                   (64 x 64 x 16, lower-triangular: zero k-steps skipped)
//   P3  all warps: S' = S exp(gc_last) + k^T (e v_new)    (128 x 64 x 16, one 16-row tile per warp; e_i = exp(gc_last - gc_i);
//                                                          k is exact in tf32: two mma per tile instead of three)
// The state slice lives in registers as the f32 accumulator fragment of P3 from chunk to chunk (no precision is lost to
// the operand split); shared memory holds its hi / lo split as the B operand of the next chunk's P1, and v_new likewise.
// The left operands are plain copies of what the chunk-local kernel wrote, in the layout it wrote them.  A ninth warp brings
// them in with five bulk copies per chunk (completion counted on an mbarrier): group 1 = {kcd, qs, vprime slice}, group 2 =
// {ks, aqk}, each refilled as soon as the eight compute warps have released its buffers; no compute warp issues a copy.
constexpr int SCAN_CONS = 256;              // compute threads
constexpr int SCAN_THREADS = SCAN_CONS + 32;
constexpr int SCAN_LDB = SCAN_VW + 8;       // B operands (state and v_new, hi and lo): bank = 24 t + g
constexpr int CHUNK_SCAN_SMEM = (2 * DN_CHUNK * SCAN_LDA + DN_CHUNK * SCAN_LDT + DN_CHUNK * SCAN_LDQ + DN_CHUNK + DN_CHUNK * SCAN_VW +
                                 2 * DN_K * SCAN_LDB + 4 * DN_CHUNK * SCAN_LDB) * 4 + 64;
constexpr uint32_t SCAN_G1_BYTES = DN_CHUNK * (2 * SCAN_LDA + SCAN_VW) * 4, SCAN_G2_BYTES = DN_CHUNK * (SCAN_LDT + SCAN_LDQ + 1) * 4;
constexpr unsigned SCAN_WAIT_LIMIT = 1u << 26;      // a bounded wait: a copy that never lands ends the loop instead of hanging

__device__ __forceinline__ void scan_wait(uint32_t bar, uint32_t parity, int* err) {
    unsigned it = 0;
    while (!mbar_try_wait(bar, parity))
        if (++it >= SCAN_WAIT_LIMIT) { atomicCAS(err, 0, (int)ERR_BARRIER_TIMEOUT); return; }
}
__device__ __forceinline__ void scan_cons_sync() { asm volatile("bar.sync 1, %0;" ::"n"(SCAN_CONS) : "memory"); }

static __global__ void __launch_bounds__(SCAN_THREADS) pf_dn_chunk_scan_kernel(const ChunkScratch* __restrict__ scratch, bf16* __restrict__ core_out,
                                                                        float* __restrict__ state_out, int S, int nchunks, int* __restrict__ err) {
    pdl_wait();
    extern __shared__ __align__(16) float sm[];
    float* skcd = sm;                                   // [64][SCAN_LDA]
    float* sq = skcd + DN_CHUNK * SCAN_LDA;             // [64][SCAN_LDA]
    float* sk = sq + DN_CHUNK * SCAN_LDA;               // [64][SCAN_LDT]
    float* sa = sk + DN_CHUNK * SCAN_LDT;               // [64][SCAN_LDQ]
    float* skd = sa + DN_CHUNK * SCAN_LDQ;              // [64] exp(gc_last - gc_i), lands with aqk
    float* svp = skd + DN_CHUNK;                        // [64][16]
    uint32_t* sth = reinterpret_cast<uint32_t*>(svp + DN_CHUNK * SCAN_VW);   // [128][SCAN_LDB] state, tf32 hi
    uint32_t* stl = sth + DN_K * SCAN_LDB;                                   //                  state, tf32 lo
    uint32_t* vnh = stl + DN_K * SCAN_LDB;                                   // [64][SCAN_LDB]  v_new, tf32 hi
    uint32_t* vnl = vnh + DN_CHUNK * SCAN_LDB;                               //                  v_new, tf32 lo
    uint32_t* vkh = vnl + DN_CHUNK * SCAN_LDB;                               // [64][SCAN_LDB]  v_new with row i scaled by kdec_i, hi
    uint32_t* vkl = vkh + DN_CHUNK * SCAN_LDB;                               //                  and lo
    u64* bars = reinterpret_cast<u64*>(vkl + DN_CHUNK * SCAN_LDB);           // full1, full2, empty1, empty2
    const int h = blockIdx.x, vs = blockIdx.y, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, t4 = lane & 3;
    const int v0 = vs * SCAN_VW;
    const uint32_t full1 = smem_u32(bars), full2 = smem_u32(bars + 1), empty1 = smem_u32(bars + 2), empty2 = smem_u32(bars + 3);
    if (tid == 0) {
        mbar_init(full1, 1); mbar_init(full2, 1);
        mbar_init(empty1, SCAN_CONS / 32); mbar_init(empty2, SCAN_CONS / 32);     // one arrival per compute warp
        mbar_fence_init();
    }
    for (int e = tid; e < 2 * DN_K * SCAN_LDB; e += SCAN_THREADS) sth[e] = 0u;          // state = 0 (hi and lo)
    __syncthreads();

    if (warp == SCAN_CONS / 32) {
        // ---- producer warp (one lane issues) ----
        for (int c = 0; c < nchunks; ++c) {
            const ChunkScratch& in = scratch[(size_t)h * nchunks + c];
            if (lane == 0) {
                if (c > 0) scan_wait(empty1, (c - 1) & 1, err);
                mbar_arrive_expect_tx(full1, SCAN_G1_BYTES);
                bulk_load_1d(smem_u32(skcd), &in.kcd[0][0], DN_CHUNK * SCAN_LDA * 4, full1);
                bulk_load_1d(smem_u32(sq), &in.qs[0][0], DN_CHUNK * SCAN_LDA * 4, full1);
                bulk_load_1d(smem_u32(svp), &in.vprime[vs][0][0], DN_CHUNK * SCAN_VW * 4, full1);
                if (c > 0) scan_wait(empty2, (c - 1) & 1, err);
                mbar_arrive_expect_tx(full2, SCAN_G2_BYTES);
                bulk_load_1d(smem_u32(sk), &in.ks[0][0], DN_CHUNK * SCAN_LDT * 4, full2);
                bulk_load_1d(smem_u32(sa), &in.aqk[0][0], DN_CHUNK * (SCAN_LDQ + 1) * 4, full2);      // aqk and kdec
            }
        }
        return;
    }

    // this warp's 16 x 16 piece of the state (rows = keys 16 warp .., columns = the slice's 16 values), f32, in registers
    float st[2][4];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int r = 0; r < 4; ++r) st[nt][r] = 0.f;

    for (int c = 0; c < nchunks; ++c) {
        const int t0 = c * DN_CHUNK;
        const float dec = scratch[(size_t)h * nchunks + c].eg_last[0];
        scan_wait(full1, c & 1, err);                                       // group 1 of this chunk has landed
        // ---- P1: VP = kcd S (warps 0-3), IT = qs S (warps 4-7) ----
        const int mt = warp & 3, m0 = mt * 16;
        float acc[2][4];
        {
            // two halves of the k range x three terms: six independent accumulator chains per column tile
            float a3[2][2][3][4];
#pragma unroll
            for (int i = 0; i < 48; ++i) a3[i / 24][(i / 12) & 1][(i >> 2) % 3][i & 3] = 0.f;
            const float* A = (warp < 4) ? skcd : sq;
#pragma unroll 2
            for (int k0 = 0; k0 < DN_K / 2; k0 += 8) {
#pragma unroll
                for (int hf = 0; hf < 2; ++hf) {
                    const int kk = k0 + hf * (DN_K / 2);
                    uint32_t ah[4], al[4];
                    load_a_split(A, SCAN_LDA, m0, kk, ah, al);
#pragma unroll
                    for (int nt = 0; nt < 2; ++nt) {
                        const int bi0 = (kk + t4) * SCAN_LDB + nt * 8 + g, bi1 = bi0 + 4 * SCAN_LDB;
                        mma_3xtf32_terms(a3[hf][nt], ah, al, sth[bi0], sth[bi1], stl[bi0], stl[bi1]);
                    }
                }
            }
#pragma unroll
            for (int nt = 0; nt < 2; ++nt)
#pragma unroll
                for (int r = 0; r < 4; ++r) acc[nt][r] = sum_terms(a3[0][nt], r) + sum_terms(a3[1][nt], r);
        }
        if (warp < 4) {
            // v_new = vprime - VP, stored split as the B operand of P2, and with row i scaled by exp(gc_last - gc_i) as the
            // B operand of P3 (the scale arrives with group 2, requested a chunk ago)
            scan_wait(full2, c & 1, err);
#pragma unroll
            for (int nt = 0; nt < 2; ++nt)
#pragma unroll
                for (int r = 0; r < 4; ++r) {
                    const int row = m0 + g + 8 * (r >> 1), col = nt * 8 + 2 * t4 + (r & 1);
                    const float vn = svp[row * SCAN_VW + col] - acc[nt][r];
                    uint32_t hi, lo;
                    tf32_split(vn, hi, lo);
                    vnh[row * SCAN_LDB + col] = hi;
                    vnl[row * SCAN_LDB + col] = lo;
                    tf32_split(vn * skd[row], hi, lo);
                    vkh[row * SCAN_LDB + col] = hi;
                    vkl[row * SCAN_LDB + col] = lo;
                }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(empty1, 1);                         // this warp is done with kcd / qs / vprime
        scan_cons_sync();                                              // v_new complete
        scan_wait(full2, c & 1, err);                                       // group 2 of this chunk has landed
        // ---- P2 (warps 4-7): out = IT + aqk v_new; aqk is lower triangular, so row tile mt needs tokens j < 16 (mt + 1) only ----
        if (warp >= 4) {
            float a3[2][3][4];
#pragma unroll
            for (int i = 0; i < 24; ++i) a3[i / 12][(i >> 2) % 3][i & 3] = 0.f;
            for (int k0 = 0; k0 < 16 * (mt + 1); k0 += 8) {
                uint32_t ah[4], al[4];
                load_a_split(sa, SCAN_LDQ, m0, k0, ah, al);
#pragma unroll
                for (int nt = 0; nt < 2; ++nt) {
                    const int bi0 = (k0 + t4) * SCAN_LDB + nt * 8 + g, bi1 = bi0 + 4 * SCAN_LDB;
                    mma_3xtf32_terms(a3[nt], ah, al, vnh[bi0], vnh[bi1], vnl[bi0], vnl[bi1]);
                }
            }
#pragma unroll
            for (int nt = 0; nt < 2; ++nt)
#pragma unroll
                for (int r = 0; r < 4; ++r) acc[nt][r] += sum_terms(a3[nt], r);
#pragma unroll
            for (int nt = 0; nt < 2; ++nt)
#pragma unroll
                for (int hr = 0; hr < 2; ++hr) {
                    const int tok = t0 + m0 + g + 8 * hr;
                    if (tok < S) {
                        bf16* dst = core_out + (size_t)tok * DN_V_SIZE + h * DN_V + v0 + nt * 8 + 2 * t4;
                        *reinterpret_cast<__nv_bfloat162*>(dst) = __halves2bfloat162(f2bf(acc[nt][2 * hr]), f2bf(acc[nt][2 * hr + 1]));
                    }
                }
        }
        // ---- P3 (all warps): S' = S exp(gc_last) + k^T (e v_new); this warp owns state rows (keys) 16 warp .. 16 warp + 15 ----
        {
            const int d0 = warp * 16;
            // k is exact in tf32, so each tile takes two mma (k x lo, k x hi of the scaled v_new) on separate accumulators
            float a2[2][2][2][4];
#pragma unroll
            for (int i = 0; i < 32; ++i) a2[i >> 4][(i >> 3) & 1][(i >> 2) & 1][i & 3] = 0.f;
#pragma unroll 2
            for (int k0 = 0; k0 < DN_CHUNK / 2; k0 += 8) {
#pragma unroll
                for (int hf = 0; hf < 2; ++hf) {
                    const int kk = k0 + hf * (DN_CHUNK / 2);
                    uint32_t a[4];
                    load_at_exact(sk, SCAN_LDT, d0, kk, a);
#pragma unroll
                    for (int nt = 0; nt < 2; ++nt) {
                        const int bi0 = (kk + t4) * SCAN_LDB + nt * 8 + g, bi1 = bi0 + 4 * SCAN_LDB;
                        mma_tf32(a2[hf][nt][0], a, vkl[bi0], vkl[bi1]);
                        mma_tf32(a2[hf][nt][1], a, vkh[bi0], vkh[bi1]);
                    }
                }
            }
#pragma unroll
            for (int nt = 0; nt < 2; ++nt)
#pragma unroll
                for (int r = 0; r < 4; ++r)
                    st[nt][r] = fmaf(st[nt][r], dec, (a2[0][nt][0][r] + a2[1][nt][0][r]) + (a2[0][nt][1][r] + a2[1][nt][1][r]));
            // the new state, split, for the next chunk's P1 (only this warp reads or writes these rows before the barrier)
#pragma unroll
            for (int nt = 0; nt < 2; ++nt)
#pragma unroll
                for (int r = 0; r < 4; ++r) {
                    const int row = d0 + g + 8 * (r >> 1), col = nt * 8 + 2 * t4 + (r & 1);
                    uint32_t hi, lo;
                    tf32_split(st[nt][r], hi, lo);
                    sth[row * SCAN_LDB + col] = hi;
                    stl[row * SCAN_LDB + col] = lo;
                }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(empty2, 1);                         // this warp is done with aqk / ks
        scan_cons_sync();                                              // the new state split is complete; v_new may be overwritten
    }
    // final state in the reference layout [head][v][k], from the f32 registers
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            const int d = warp * 16 + g + 8 * (r >> 1), v = nt * 8 + 2 * t4 + (r & 1);
            state_out[((size_t)h * DN_V + v0 + v) * DN_K + d] = st[nt][r];
        }
}

// ---- gated RMSNorm of the DeltaNet output: one warp per (token, head) --------------------------------
static __global__ void __launch_bounds__(256) pf_gated_norm_kernel(const bf16* __restrict__ core, const bf16* __restrict__ proj, int ldp,
                                                            const bf16* __restrict__ norm_w, bf16* __restrict__ out, int S) {
    pdl_wait();
    const int gw = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (gw >= S * DN_HEADS) return;
    const int t = gw / DN_HEADS, h = gw % DN_HEADS;
    const uint2 orw = *(reinterpret_cast<const uint2*>(core + (size_t)t * DN_V_SIZE + h * DN_V) + lane);
    const uint2 zrw = *(reinterpret_cast<const uint2*>(proj + (size_t)t * ldp + DN_CONV_CH + h * DN_V) + lane);
    const uint2 nrw = __ldg(reinterpret_cast<const uint2*>(norm_w) + lane);
    const float ov[4] = {bf_lo(orw.x), bf_hi(orw.x), bf_lo(orw.y), bf_hi(orw.y)};
    const float zv[4] = {bf_lo(zrw.x), bf_hi(zrw.x), bf_lo(zrw.y), bf_hi(zrw.y)};
    const float nw[4] = {bf_lo(nrw.x), bf_hi(nrw.x), bf_lo(nrw.y), bf_hi(nrw.y)};
    const float var = warp_sum(ov[0] * ov[0] + ov[1] * ov[1] + ov[2] * ov[2] + ov[3] * ov[3]) * (1.0f / DN_V);
    const float r = rsqrt_ieee(var + RMS_EPS);
    float u[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) u[i] = rbf(nw[i] * rbf(ov[i] * r)) * silu_f(zv[i]);
    bf16* dst = out + (size_t)t * DN_V_SIZE + h * DN_V + lane * 4;
    *reinterpret_cast<__nv_bfloat162*>(dst) = __halves2bfloat162(f2bf(u[0]), f2bf(u[1]));
    *reinterpret_cast<__nv_bfloat162*>(dst + 2) = __halves2bfloat162(f2bf(u[2]), f2bf(u[3]));
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
