// Batched greedy decode: B independent sequences per GPU advance one token per call, weights read once per
// step for all of them.  The reference is batch-1 only (models/qwen35_0p8b/README.md:167); this is the
// additive op its benchmark configuration "64 sequences per GPU, 2048-token contexts" needs.  Every sequence
// follows exactly the bs=1 arithmetic of the decode megakernel (kernel.cu:409-741 restated), so the CPU oracle
// for a sequence is the bs=1 oracle.
//
// One step = a short stream of kernels (no host synchronisation, capturable in a CUDA graph):
//   per layer  RMSNorm rows -> projection GEMM (tcgen05, M = B) -> DeltaNet step (conv + SiLU, L2 norm,
//              recurrence on the f32 state of every (sequence, head)) + conv shift + gated norm, or q/k norm +
//              RoPE + paged KV append + attention over the paged bf16 KV cache -> output GEMM + residual ->
//              RMSNorm -> gate/up GEMM with fused SiLU*up -> down GEMM + residual
//   finally    RMSNorm -> LM-head GEMM [B, 248320] -> per-row arg-max (lowest index among equal bf16 maxima)
// KV cache pages: [layer 6][page][kv head 2][64 positions][256] bf16, addressed through block_table[B][max_pages].
#include <cuda.h>

#include "prefill_kernels.cuh"

#include <cmath>
#include <mutex>

#include "runtime.h"

namespace q35 {
bool make_tmap(CUtensorMap* tm, const void* ptr, int rows, int cols, int ld, int box_rows);      // gemm_tcgen05.cu


int gemm_bf16(const bf16* A, int lda, const bf16* B, int b_rows, bf16* C, int ldc, const bf16* R, int ldr,
              int M, int N, int K, int epi, int up_row_offset, cudaStream_t stream);

constexpr int KV_PAGE = 64;

__device__ __forceinline__ float conv_silu4(const bf16* conv_w, int ch, float4 st, float x) {
    const uint2 wr = __ldg(reinterpret_cast<const uint2*>(conv_w) + ch);
    float c = bf_lo(wr.x) * st.y;
    c = fmaf(bf_hi(wr.x), st.z, c);
    c = fmaf(bf_lo(wr.y), st.w, c);
    c = fmaf(bf_hi(wr.y), x, c);
    return rbf(silu_f(rbf(c)));
}

// ---- DeltaNet step: one CTA (256 threads) per (sequence, head, block of 64 value rows) -------------------
constexpr int BD_DN_ROWS = 64;
__global__ void __launch_bounds__(256) bd_dn_step_kernel(const bf16* __restrict__ proj, int ldp, const bf16* __restrict__ conv_w,
                                                         const bf16* __restrict__ a_log, const bf16* __restrict__ dt_bias,
                                                         const float* __restrict__ conv, size_t conv_seq_stride,
                                                         float* __restrict__ state, size_t state_seq_stride, bf16* __restrict__ core_out) {
    pdl_wait();
    __shared__ __align__(16) float sqk[2][DN_K];
    __shared__ float red[2][4];
    __shared__ float shd[2];
    __shared__ float svv[BD_DN_ROWS];
    const int b = blockIdx.x, h = blockIdx.y, rb = blockIdx.z, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const bf16* xrow = proj + (size_t)b * ldp;
    const float4* cv = reinterpret_cast<const float4*>(conv + (size_t)b * conv_seq_stride);
    // this warp's state rows first: they depend on nothing computed here, so they stream in while q, k, v, beta and the decay
    // are prepared (the kernel is bound by these 134 MB per launch)
    float* st_base = state + (size_t)b * state_seq_stride + (size_t)h * DN_V * DN_K;
    constexpr int RPW = BD_DN_ROWS / 8;                 // rows per warp
    float4 t[RPW];
#pragma unroll
    for (int r = 0; r < RPW; ++r)
        t[r] = __ldcs(reinterpret_cast<const float4*>(st_base + (size_t)(rb * BD_DN_ROWS + warp * RPW + r) * DN_K) + lane);
    // q (threads 0-127) and k (threads 128-255) of this head: conv + SiLU, then the L2 norm in bf16 arithmetic
    const int which = tid >> 7, i = tid & 127;
    const int chx = which * DN_QK_SIZE + h * DN_K + i;
    const float cx = conv_silu4(conv_w, chx, cv[chx], bf2f(xrow[chx]));
    const float s0 = warp_sum(rbf(cx * cx));
    if (lane == 0) red[which][warp & 3] = s0;
    if (tid < BD_DN_ROWS) {
        const int ch = 2 * DN_QK_SIZE + h * DN_V + rb * BD_DN_ROWS + tid;
        svv[tid] = conv_silu4(conv_w, ch, cv[ch], bf2f(xrow[ch]));
    }
    if (tid == 0) {
        const float bb = bf2f(xrow[DN_CONV_CH + DN_V_SIZE + h]);
        const float aa = bf2f(xrow[DN_CONV_CH + DN_V_SIZE + DN_HEADS + h]);
        const float x = aa + bf2f(dt_bias[h]);
        const float sp = (x > 20.f) ? x : log1pf(expf(x));
        shd[0] = rbf(sigmoid_f(bb));
        shd[1] = expf(-expf(bf2f(a_log[h])) * sp);
    }
    __syncthreads();
    {
        float t = ((red[which][0] + red[which][1]) + red[which][2]) + red[which][3];
        t = rbf(rbf(t) + 1e-6f);
        const float n = rbf(cx * rbf(1.0f / rbf(sqrtf(t))));
        sqk[which][i] = which ? n : n * 0.08838834764831845f;
    }
    __syncthreads();
    const float4 q4 = *reinterpret_cast<const float4*>(&sqk[0][lane * 4]);
    const float4 k4 = *reinterpret_cast<const float4*>(&sqk[1][lane * 4]);
    const float beta = shd[0], decay = shd[1];
#pragma unroll
    for (int r = 0; r < RPW; ++r) {
        const int vl = warp * RPW + r, v = rb * BD_DN_ROWS + vl;
        float4 u = t[r];
        u.x = __fmul_rn(u.x, decay); u.y = __fmul_rn(u.y, decay); u.z = __fmul_rn(u.z, decay); u.w = __fmul_rn(u.w, decay);
        float kv = __fadd_rn(__fadd_rn(__fadd_rn(__fmul_rn(u.x, k4.x), __fmul_rn(u.y, k4.y)), __fmul_rn(u.z, k4.z)), __fmul_rn(u.w, k4.w));
        kv = warp_sum(kv);
        const float delta = __fmul_rn(__fsub_rn(svv[vl], kv), beta);
        u.x = __fadd_rn(u.x, __fmul_rn(k4.x, delta)); u.y = __fadd_rn(u.y, __fmul_rn(k4.y, delta));
        u.z = __fadd_rn(u.z, __fmul_rn(k4.z, delta)); u.w = __fadd_rn(u.w, __fmul_rn(k4.w, delta));
        float o = __fadd_rn(__fadd_rn(__fadd_rn(__fmul_rn(u.x, q4.x), __fmul_rn(u.y, q4.y)), __fmul_rn(u.z, q4.z)), __fmul_rn(u.w, q4.w));
        o = warp_sum(o);
        __stcs(reinterpret_cast<float4*>(st_base + (size_t)v * DN_K) + lane, u);
        if (lane == 0) core_out[(size_t)b * DN_V_SIZE + h * DN_V + v] = f2bf(o);
    }
}

// conv window shift for every (sequence, channel), after all readers of the old window have finished
__global__ void bd_conv_shift_kernel(const bf16* __restrict__ proj, int ldp, float* __restrict__ conv, size_t conv_seq_stride, int B) {
    pdl_wait();
    const int idx = blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= B * DN_CONV_CH) return;
    const int b = idx / DN_CONV_CH, ch = idx % DN_CONV_CH;
    float4* p = reinterpret_cast<float4*>(conv + (size_t)b * conv_seq_stride) + ch;
    const float4 s = *p;
    *p = make_float4(s.y, s.z, s.w, bf2f(proj[(size_t)b * ldp + ch]));
}

__device__ __forceinline__ bool bd_pos_ok(int pos, int max_ctx) { return pos >= 0 && pos < max_ctx; }

__device__ __forceinline__ bf16* kv_row(bf16* pages, const int* table, int max_pages, int b, int kvh, int pos) {
    const int page = table[b * max_pages + pos / KV_PAGE];
    return pages + (((size_t)page * FA_KV_HEADS + kvh) * KV_PAGE + (pos % KV_PAGE)) * FA_HEAD_DIM;
}

// ---- attention preparation: one warp per (sequence, slot); slots 0-7 q heads, 8-9 k heads, 10-11 v heads ----
__global__ void __launch_bounds__(256) bd_qk_norm_rope_kernel(const bf16* __restrict__ proj, int ldp, const bf16* __restrict__ qn_w,
                                                              const bf16* __restrict__ kn_w, const RopeTable inv_freq,
                                                              const int* __restrict__ positions, const int* __restrict__ table, int max_pages,
                                                              bf16* __restrict__ q_out, bf16* __restrict__ k_pages, bf16* __restrict__ v_pages, int B,
                                                              int max_ctx, int* __restrict__ err) {
    pdl_wait();
    const int gw = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (gw >= B * 12) return;
    const int b = gw / 12, slot = gw % 12, pos = positions[b];
    // A sequence whose position left [0, max_ctx) would index the block table beyond its row and the score scratch beyond
    // max_ctx.  Positions advance on the device, so the check is here: the row is skipped (no K/V write, its attention
    // output is zero, its position stops advancing) and the sticky status word reports a bad argument.
    if (!bd_pos_ok(pos, max_ctx)) {
        if (lane == 0 && slot == 0) atomicCAS(err, 0, (int)ERR_BAD_ARG);
        return;
    }
    if (slot >= 10) {
        const int kvh = slot - 10;
        const uint4 v = *(reinterpret_cast<const uint4*>(proj + (size_t)b * ldp + FA_QPROJ + FA_KV_SIZE + kvh * FA_HEAD_DIM) + lane);
        *(reinterpret_cast<uint4*>(kv_row(v_pages, table, max_pages, b, kvh, pos)) + lane) = v;
        return;
    }
    const bool isq = slot < 8;
    const bf16* src = proj + (size_t)b * ldp + (isq ? slot * 2 * FA_HEAD_DIM : FA_QPROJ + (slot - 8) * FA_HEAD_DIM);
    const bf16* nw = isq ? qn_w : kn_w;
    float xv[8], ss = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) { xv[i] = bf2f(src[lane + 32 * i]); ss += xv[i] * xv[i]; }
    const float r = rsqrt_ieee(warp_sum(ss) * (1.0f / FA_HEAD_DIM) + RMS_EPS);
#pragma unroll
    for (int i = 0; i < 8; ++i) xv[i] = rbf((xv[i] * r) * (1.0f + bf2f(nw[lane + 32 * i])));
    const float ang = (float)pos * inv_freq.f[lane];
    const float cs = rbf(cosf(ang)), sn = rbf(sinf(ang));
    const float x1 = xv[0], x2 = xv[1];
    xv[0] = rbf(rbf(x1 * cs) + rbf(-x2 * sn));
    xv[1] = rbf(rbf(x2 * cs) + rbf(x1 * sn));
    bf16* dst = isq ? q_out + (size_t)b * FA_Q_SIZE + slot * FA_HEAD_DIM : kv_row(k_pages, table, max_pages, b, slot - 8, pos);
#pragma unroll
    for (int i = 0; i < 8; ++i) dst[lane + 32 * i] = f2bf(xv[i]);
}

// ---- decode attention over the paged cache, split over the context -----------------------------------------
// Three kernels per layer keep the bf16 rounding points of the bs=1 path (P is rounded with the global normaliser):
//   scores  one CTA per (sequence, kv head, slice z of Z): walks the 64-position pages z, z + Z, ... of the sequence;
//           bf16(q.k)/16 for the four q heads of the kv head (K row read once, coalesced) to global memory, running
//           maximum and sum-exp per head over the slice
//   pv      same grid: global max / normaliser from the Z slice statistics, P = bf16(exp(s-m)/l), P.V accumulated over the
//           slice's pages in registers, one partial per slice
//   merge   one warp per (sequence, q head): sum of the slice partials in order, bf16, times bf16(sigmoid(gate))
// A CTA reads its page ids once and keeps the next two pages' rows in flight (cp.async, three buffers) while it computes on
// the current one: the chain position -> page id -> rows is paid once per slice, not once per 128 positions.
constexpr int BD_CHUNK = KV_PAGE;                        // positions per step of a slice: one page
constexpr int BD_MAX_PAGES_SLICE = 128;                  // page ids a CTA keeps in shared memory

__device__ __forceinline__ const bf16* kv_row_c(const bf16* pages, const int* tb, int kvh, int pos) {
    return pages + (((size_t)tb[pos / KV_PAGE] * FA_KV_HEADS + kvh) * KV_PAGE + (pos % KV_PAGE)) * FA_HEAD_DIM;
}

// Both kernels receive a page's K (or V) rows by TMA: the page pool of a layer is a 2-D bf16 tensor [pages x kv heads x 64
// rows][256], a page of one kv head arrives as four boxes of 64 rows x 64 dimensions in the 128-byte-swizzled layout (row r
// of a box at r x 128 bytes, its 16-byte pieces XORed with r mod 8), which ldmatrix reads without bank conflicts.  One
// thread issues the four copies of a page on an mbarrier; three page buffers keep two pages in flight while the four warps
// run mma.sync m16n8k16 tiles on the third: the M side holds the four q heads of the kv head (rows 4-15 of the tile are
// zero), so a position costs a handful of instructions instead of a warp reduction per head.  (The first form staged rows
// with cp.async, 16 per thread and page: the issue rate of those copies, not the bytes in flight, bounded it at 3.5 TB/s.)
constexpr int BD_LD = FA_HEAD_DIM + 8;                   // shared-memory row of the Q tile, bf16 elements
constexpr int BD_PLD = BD_CHUNK + 8;
constexpr int BD_NBUF = 3;                               // page buffers per CTA
constexpr int BD_PAGE_BYTES = KV_PAGE * FA_HEAD_DIM * 2; // 32 KB: four 8 KB boxes
constexpr int BD_SC_SMEM = 1024 + BD_NBUF * BD_PAGE_BYTES + 16 * BD_LD * 2;
constexpr int BD_PV_SMEM = 1024 + BD_NBUF * BD_PAGE_BYTES + 16 * BD_PLD * 2;
constexpr unsigned BD_WAIT_LIMIT = 1u << 24;

// byte offset of element (row, dim) of a page buffer (four boxes of 64 dims; 128-byte rows; 16-byte pieces swizzled)
__device__ __forceinline__ uint32_t bd_page_off(int row, int dim) {
    return (uint32_t)((dim >> 6) * (KV_PAGE * 128) + row * 128 + ((((dim & 63) >> 3) ^ (row & 7)) << 4) + (dim & 7) * 2);
}
// one thread: the four copies of page `page` of kv head `kvh` into buffer `dst` (shared address), counted on `bar`
__device__ __forceinline__ void bd_issue_page(const void* tmap, int page, int kvh, uint32_t dst, uint32_t bar) {
    mbar_arrive_expect_tx(bar, BD_PAGE_BYTES);
    const int y = (page * FA_KV_HEADS + kvh) * KV_PAGE;
#pragma unroll
    for (int t = 0; t < 4; ++t) tma_load_2d(dst + t * (KV_PAGE * 128), tmap, t * 64, y, bar);
}
// bounded wait for a page; a wait that runs out sets the status word and the kernel carries on to its end
__device__ __forceinline__ void bd_wait_bar(uint32_t bar, uint32_t parity, int* status) {
    unsigned it = 0;
    while (!mbar_try_wait(bar, parity))
        if (++it >= BD_WAIT_LIMIT) { atomicCAS(status, 0, (int)ERR_BARRIER_TIMEOUT); return; }
}

__global__ void __launch_bounds__(128) bd_att_scores_kernel(const __grid_constant__ CUtensorMap tmK, const bf16* __restrict__ q,
                                                            const int* __restrict__ positions, const int* __restrict__ table, int max_pages,
                                                            float* __restrict__ scores, float* __restrict__ stats, int max_ctx, int max_slices,
                                                            int* __restrict__ status) {
    extern __shared__ unsigned char bd_sm_raw[];
    __shared__ float ssc[2][FA_GQA][BD_CHUNK];           // scores of a page, double buffered: one barrier per page
    __shared__ int spg[BD_MAX_PAGES_SLICE];
    __shared__ __align__(8) u64 bars[BD_NBUF];
    const uint32_t raw = smem_u32(bd_sm_raw), pages_s = (raw + 1023u) & ~1023u;      // swizzled boxes need 1024-byte alignment
    unsigned char* pages_p = bd_sm_raw + (pages_s - raw);
    bf16* Qs = reinterpret_cast<bf16*>(pages_p + BD_NBUF * BD_PAGE_BYTES);             // [16][BD_LD], rows 0-3 = the q heads of this kv head
    const int b = blockIdx.x, kvh = blockIdx.y, z = blockIdx.z, Z = gridDim.z, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (tid == 0) {
        asm volatile("prefetch.tensormap [%0];" ::"l"(&tmK) : "memory");
        for (int i = 0; i < BD_NBUF; ++i) mbar_init(smem_u32(&bars[i]), 1);
        mbar_fence_init();
    }
    pdl_wait();
    const int L = positions[b] + 1;
    const int npages = (L + KV_PAGE - 1) / KV_PAGE;
    if (!bd_pos_ok(L - 1, max_ctx) || z >= npages) return;
    const int mine = (npages - z + Z - 1) / Z;           // pages z, z + Z, ...
    const int* tb = table + b * max_pages;
    for (int i = tid; i < mine && i < BD_MAX_PAGES_SLICE; i += 128) spg[i] = tb[z + i * Z];
    for (int i = tid; i < 16 * (FA_HEAD_DIM / 8); i += 128) {
        const int r = i / (FA_HEAD_DIM / 8), c8 = i % (FA_HEAD_DIM / 8);
        uint4 v = make_uint4(0, 0, 0, 0);
        if (r < FA_GQA) v = *reinterpret_cast<const uint4*>(q + (size_t)b * FA_Q_SIZE + (kvh * FA_GQA + r) * FA_HEAD_DIM + c8 * 8);
        *reinterpret_cast<uint4*>(Qs + r * BD_LD + c8 * 8) = v;
    }
    __syncthreads();
    if (tid == 0) {
        bd_issue_page(&tmK, spg[0], kvh, pages_s, smem_u32(&bars[0]));
        if (mine > 1) bd_issue_page(&tmK, spg[1], kvh, pages_s + BD_PAGE_BYTES, smem_u32(&bars[1]));
    }
    // the Q fragments of all 16 k-steps stay in registers
    uint32_t qf[FA_HEAD_DIM / 16][4];
#pragma unroll
    for (int ks = 0; ks < FA_HEAD_DIM / 16; ++ks) ldsm_x4(qf[ks], Qs + (lane & 15) * BD_LD + ks * 16 + (lane >> 4) * 8);
    float run_m = -INFINITY, run_s = 0.f;                 // warp g: head g's statistics over the slice
    for (int i = 0; i < mine; ++i) {
        const int j0 = (z + i * Z) * KV_PAGE, cn = min(KV_PAGE, L - j0);
        const uint32_t Kc = pages_s + (i % BD_NBUF) * BD_PAGE_BYTES;
        // buffer (i + 2) % 3 was read in step i - 1; every warp has passed that step's barrier after its MMAs
        if (tid == 0 && i + 2 < mine) bd_issue_page(&tmK, spg[i + 2], kvh, pages_s + ((i + 2) % BD_NBUF) * BD_PAGE_BYTES, smem_u32(&bars[(i + 2) % BD_NBUF]));
        bd_wait_bar(smem_u32(&bars[i % BD_NBUF]), (uint32_t)((i / BD_NBUF) & 1), status);
        // warp w: keys [16w, 16w+16) = 2 tiles of 8 keys; even and odd k-steps on separate accumulators (two chains of 8)
        float acc[2][2][4];
#pragma unroll
        for (int e = 0; e < 16; ++e) acc[e >> 3][(e >> 2) & 1][e & 3] = 0.f;
        const int krow = warp * 16 + (lane & 7) + 8 * (lane >> 4);
        float (*sp)[BD_CHUNK] = ssc[i & 1];
#pragma unroll
        for (int ks = 0; ks < FA_HEAD_DIM / 16; ++ks) {
            uint32_t bb[4];
            const uint32_t baddr = Kc + bd_page_off(krow, ks * 16 + 8 * ((lane >> 3) & 1));
            asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];" : "=r"(bb[0]), "=r"(bb[1]), "=r"(bb[2]), "=r"(bb[3]) : "r"(baddr));
            mma_16816(acc[ks & 1][0], qf[ks], bb[0], bb[1]);
            mma_16816(acc[ks & 1][1], qf[ks], bb[2], bb[3]);
        }
        {   // accumulator rows 0-3 (g = lane/4 < 4) are the four heads; columns 2c, 2c+1 of each 8-key tile
            const int g = lane >> 2, cc = lane & 3;
            if (g < FA_GQA) {
#pragma unroll
                for (int nt = 0; nt < 2; ++nt) {
                    sp[g][warp * 16 + nt * 8 + 2 * cc] = rbf(acc[0][nt][0] + acc[1][nt][0]) * 0.0625f;
                    sp[g][warp * 16 + nt * 8 + 2 * cc + 1] = rbf(acc[0][nt][1] + acc[1][nt][1]) * 0.0625f;
                }
            }
        }
        __syncthreads();                                 // scores of the page complete; every warp is done with this buffer
        {   // warp g: statistics of head g over this page, folded into the slice's; scores to global
            const int g = warp;
            float mx = -INFINITY;
            for (int j = lane; j < cn; j += 32) mx = fmaxf(mx, sp[g][j]);
            mx = warp_max(mx);
            float sm = 0.f;
            for (int j = lane; j < cn; j += 32) sm += expf(sp[g][j] - mx);
            sm = warp_sum(sm);
            const float nm = fmaxf(run_m, mx);
            run_s = (run_m == -INFINITY ? 0.f : run_s * expf(run_m - nm)) + sm * expf(mx - nm);
            run_m = nm;
            float* dst = scores + ((size_t)b * FA_Q_HEADS + kvh * FA_GQA + g) * max_ctx + j0;
            for (int j = lane; j < cn; j += 32) dst[j] = sp[g][j];
        }
        // the other score buffer is written next; this one again two pages on, after the next page's barrier
    }
    if (lane == 0) {
        float* st = stats + (((size_t)b * FA_Q_HEADS + kvh * FA_GQA + warp) * max_slices + z) * 2;
        st[0] = run_m; st[1] = run_s;
    }
}

__global__ void __launch_bounds__(128) bd_att_pv_kernel(const __grid_constant__ CUtensorMap tmV, const int* __restrict__ positions,
                                                        const int* __restrict__ table, int max_pages, const float* __restrict__ scores,
                                                        const float* __restrict__ stats, float* __restrict__ partial, int max_ctx, int max_slices,
                                                        int* __restrict__ status) {
    extern __shared__ unsigned char bd_sm_raw[];
    __shared__ float sml[FA_GQA][2];
    __shared__ int spg[BD_MAX_PAGES_SLICE];
    __shared__ __align__(8) u64 bars[BD_NBUF];
    const uint32_t raw = smem_u32(bd_sm_raw), pages_s = (raw + 1023u) & ~1023u;
    unsigned char* pages_p = bd_sm_raw + (pages_s - raw);
    bf16* Ps = reinterpret_cast<bf16*>(pages_p + BD_NBUF * BD_PAGE_BYTES);             // [16][BD_PLD], rows 0-3 = P of the four heads
    const int b = blockIdx.x, kvh = blockIdx.y, z = blockIdx.z, Z = gridDim.z, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (tid == 0) {
        asm volatile("prefetch.tensormap [%0];" ::"l"(&tmV) : "memory");
        for (int i = 0; i < BD_NBUF; ++i) mbar_init(smem_u32(&bars[i]), 1);
        mbar_fence_init();
    }
    pdl_wait();
    const int L = positions[b] + 1;
    const int npages = (L + KV_PAGE - 1) / KV_PAGE;
    if (!bd_pos_ok(L - 1, max_ctx) || z >= npages) return;
    const int mine = (npages - z + Z - 1) / Z, nsl = min(Z, npages);
    const int* tb = table + b * max_pages;
    for (int i = tid; i < mine && i < BD_MAX_PAGES_SLICE; i += 128) spg[i] = tb[z + i * Z];
    {
        const int head = kvh * FA_GQA + warp;
        const float* st = stats + ((size_t)b * FA_Q_HEADS + head) * max_slices * 2;
        float mx = -INFINITY;
        for (int k = lane; k < nsl; k += 32) mx = fmaxf(mx, st[2 * k]);
        mx = warp_max(mx);
        float sm = 0.f;
        for (int k = lane; k < nsl; k += 32) sm += st[2 * k + 1] * expf(st[2 * k] - mx);
        sm = warp_sum(sm);
        if (lane == 0) { sml[warp][0] = mx; sml[warp][1] = sm; }
    }
    for (int i = tid; i < 12 * BD_PLD; i += 128) Ps[4 * BD_PLD + i] = f2bf(0.f);      // rows 4-15 of the P tile stay zero
    __syncthreads();
    if (tid == 0) {
        bd_issue_page(&tmV, spg[0], kvh, pages_s, smem_u32(&bars[0]));
        if (mine > 1) bd_issue_page(&tmV, spg[1], kvh, pages_s + BD_PAGE_BYTES, smem_u32(&bars[1]));
    }
    // warp w: output dims [64w, 64w+64) = 8 tiles of 8 dims (box w of a page buffer), accumulated over the slice's pages
    float acc[8][4];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) { acc[nt][0] = 0.f; acc[nt][1] = 0.f; acc[nt][2] = 0.f; acc[nt][3] = 0.f; }
    // a thread forms two P values per page (heads tid / 64 and tid / 64 + 2, position tid % 64); their scores are fetched one
    // page ahead, so the global-memory latency hides behind the MMAs of the page before
    const int pj = tid & 63, pg0 = tid >> 6;
    const float* sc0 = scores + ((size_t)b * FA_Q_HEADS + kvh * FA_GQA + pg0) * max_ctx;
    const float* sc1 = sc0 + (size_t)2 * max_ctx;
    float s_next0 = 0.f, s_next1 = 0.f;
    if (z * KV_PAGE + pj < L) { s_next0 = sc0[z * KV_PAGE + pj]; s_next1 = sc1[z * KV_PAGE + pj]; }
    for (int i = 0; i < mine; ++i) {
        const int j0 = (z + i * Z) * KV_PAGE, cn = min(KV_PAGE, L - j0);
        const uint32_t Vc = pages_s + (i % BD_NBUF) * BD_PAGE_BYTES;
        if (tid == 0 && i + 2 < mine) bd_issue_page(&tmV, spg[i + 2], kvh, pages_s + ((i + 2) % BD_NBUF) * BD_PAGE_BYTES, smem_u32(&bars[(i + 2) % BD_NBUF]));
        const float s_cur0 = s_next0, s_cur1 = s_next1;
        if (i + 1 < mine) {
            const int jn = (z + (i + 1) * Z) * KV_PAGE + pj;
            if (jn < L) { s_next0 = sc0[jn]; s_next1 = sc1[jn]; }
        }
        // P of this page while the copies fly
        Ps[pg0 * BD_PLD + pj] = f2bf(pj < cn ? rbf(expf(s_cur0 - sml[pg0][0]) / sml[pg0][1]) : 0.f);
        Ps[(pg0 + 2) * BD_PLD + pj] = f2bf(pj < cn ? rbf(expf(s_cur1 - sml[pg0 + 2][0]) / sml[pg0 + 2][1]) : 0.f);
        bd_wait_bar(smem_u32(&bars[i % BD_NBUF]), (uint32_t)((i / BD_NBUF) & 1), status);
        if (cn < KV_PAGE) {
            // rows past the sequence's end hold whatever the pool has there; P is zero for them, but 0 x NaN is not: clear them
            unsigned char* vb = pages_p + (i % BD_NBUF) * BD_PAGE_BYTES;
            for (int e = tid; e < (KV_PAGE - cn) * 32; e += 128) {
                const int r = cn + e / 32, piece = e % 32;
                *reinterpret_cast<uint4*>(vb + (piece >> 3) * (KV_PAGE * 128) + r * 128 + (piece & 7) * 16) = make_uint4(0, 0, 0, 0);
            }
        }
        __syncthreads();
        const int steps = (cn + 15) / 16;
        for (int ks = 0; ks < steps; ++ks) {
            uint32_t a[4];
            ldsm_x4(a, Ps + (lane & 15) * BD_PLD + ks * 16 + (lane >> 4) * 8);
            const int vrow = ks * 16 + (lane & 7) + 8 * ((lane >> 3) & 1);
#pragma unroll
            for (int np = 0; np < 4; ++np) {
                uint32_t bb[4];
                const uint32_t baddr = Vc + bd_page_off(vrow, warp * 64 + np * 16 + 8 * (lane >> 4));
                asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];" : "=r"(bb[0]), "=r"(bb[1]), "=r"(bb[2]), "=r"(bb[3]) : "r"(baddr));
                mma_16816(acc[2 * np], a, bb[0], bb[1]);
                mma_16816(acc[2 * np + 1], a, bb[2], bb[3]);
            }
        }
        __syncthreads();                                 // P tile and this buffer are free again
    }
    const int g = lane >> 2, cc = lane & 3;
    if (g < FA_GQA) {
        float* dst = partial + (((size_t)b * FA_Q_HEADS + kvh * FA_GQA + g) * max_slices + z) * FA_HEAD_DIM + warp * 64 + 2 * cc;
#pragma unroll
        for (int nt = 0; nt < 8; ++nt) *reinterpret_cast<float2*>(dst + nt * 8) = make_float2(acc[nt][0], acc[nt][1]);
    }
}

__global__ void __launch_bounds__(256) bd_att_merge_kernel(const float* __restrict__ partial, const int* __restrict__ positions,
                                                           const bf16* __restrict__ proj, int ldp, bf16* __restrict__ out, int B, int max_slices,
                                                           int n_slices, int max_ctx) {
    pdl_trigger();      // the out-projection GEMM loads its first weight tiles beside this kernel
    pdl_wait();
    const int gw = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (gw >= B * FA_Q_HEADS) return;
    const int b = gw / FA_Q_HEADS, head = gw % FA_Q_HEADS;
    if (!bd_pos_ok(positions[b], max_ctx)) {           // skipped sequence: a defined (zero) attention output
        *(reinterpret_cast<uint4*>(out + (size_t)b * FA_Q_SIZE + head * FA_HEAD_DIM) + lane) = make_uint4(0, 0, 0, 0);
        return;
    }
    const int nsl = min(n_slices, (positions[b] + 1 + KV_PAGE - 1) / KV_PAGE);
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    const float* pb = partial + ((size_t)b * FA_Q_HEADS + head) * max_slices * FA_HEAD_DIM + lane * 8;
    for (int c = 0; c < nsl; ++c) {
        const float4 a0 = *reinterpret_cast<const float4*>(pb + (size_t)c * FA_HEAD_DIM), a1 = *reinterpret_cast<const float4*>(pb + (size_t)c * FA_HEAD_DIM + 4);
        acc[0] += a0.x; acc[1] += a0.y; acc[2] += a0.z; acc[3] += a0.w; acc[4] += a1.x; acc[5] += a1.y; acc[6] += a1.z; acc[7] += a1.w;
    }
    const uint4 gr = *(reinterpret_cast<const uint4*>(proj + (size_t)b * ldp + head * 2 * FA_HEAD_DIM + FA_HEAD_DIM) + lane);
    const float gv[8] = {bf_lo(gr.x), bf_hi(gr.x), bf_lo(gr.y), bf_hi(gr.y), bf_lo(gr.z), bf_hi(gr.z), bf_lo(gr.w), bf_hi(gr.w)};
    uint32_t o[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const __nv_bfloat162 pr = __halves2bfloat162(f2bf(rbf(acc[2 * i]) * rbf(sigmoid_f(gv[2 * i]))),
                                                     f2bf(rbf(acc[2 * i + 1]) * rbf(sigmoid_f(gv[2 * i + 1]))));
        o[i] = *reinterpret_cast<const uint32_t*>(&pr);
    }
    *(reinterpret_cast<uint4*>(out + (size_t)b * FA_Q_SIZE + head * FA_HEAD_DIM) + lane) = make_uint4(o[0], o[1], o[2], o[3]);
}

// ---- per-row arg-max over bf16 logits [B, VOCAB]: one CTA per row ---------------------------------------
__global__ void __launch_bounds__(1024) bd_argmax_kernel(const bf16* __restrict__ logits, int* __restrict__ out_tokens, int* __restrict__ positions, int max_ctx) {
    pdl_wait();
    __shared__ float sv[32];
    __shared__ int si[32];
    const int b = blockIdx.x, tid = threadIdx.x;
    const uint4* row = reinterpret_cast<const uint4*>(logits + (size_t)b * VOCAB);
    float best = -INFINITY;
    int best_i = 0x7fffffff;
    for (int c = tid; c < VOCAB / 8; c += 1024) {
        const uint4 v = row[c];
        const float f[8] = {bf_lo(v.x), bf_hi(v.x), bf_lo(v.y), bf_hi(v.y), bf_lo(v.z), bf_hi(v.z), bf_lo(v.w), bf_hi(v.w)};
#pragma unroll
        for (int k = 0; k < 8; ++k) if (f[k] > best) { best = f[k]; best_i = c * 8 + k; }
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
        // a sequence that is already outside [0, max_ctx) was skipped by this step and stays where it is
        if (tid == 0) { out_tokens[b] = best_i; if (positions && bd_pos_ok(positions[b], max_ctx)) positions[b] += 1; }
    }
}

// debug / teacher forcing helpers
__global__ void bd_copy_rows_kernel(const bf16* __restrict__ src, bf16* __restrict__ dst, int n_u4) {
    pdl_wait();
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n_u4) reinterpret_cast<uint4*>(dst)[i] = reinterpret_cast<const uint4*>(src)[i];
}

static void* g_bscratch[64] = {};
static size_t g_bscratch_bytes[64] = {};
static std::mutex g_bscratch_mu;

static void* batched_scratch(size_t bytes) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return nullptr;
    dev &= 63;
    std::lock_guard<std::mutex> lk(g_bscratch_mu);
    if (g_bscratch_bytes[dev] < bytes) {
        if (g_bscratch[dev]) { cudaDeviceSynchronize(); cudaFree(g_bscratch[dev]); g_bscratch[dev] = nullptr; g_bscratch_bytes[dev] = 0; }
        if (cudaMalloc(&g_bscratch[dev], bytes) != cudaSuccess) { set_error("batched decode scratch allocation of %zu bytes failed", bytes); return nullptr; }
        g_bscratch_bytes[dev] = bytes;
    }
    return g_bscratch[dev];
}

typedef PrefillFused PrefillFusedB;

// upper bound of the slices per (sequence, kv head): the statistics and partial buffers are sized by it.  A slice holds at
// most BD_MAX_PAGES_SLICE page ids, so long contexts need at least pages / BD_MAX_PAGES_SLICE slices.
static int bd_max_slices(int max_ctx) {
    const int pages = (max_ctx + KV_PAGE - 1) / KV_PAGE;
    return pages < 148 ? pages : 148;
}
}  // namespace q35

static size_t batched_scratch_total(int batch, int max_ctx) {
    using namespace q35;
    const size_t rows = (size_t)batch;
    const size_t n_hidden = rows * HIDDEN, n_proj = rows * DN_PROJ_ROWS, n_att = rows * 2048, n_mlp = rows * INTER, n_logits = rows * VOCAB;
    const int max_chunks = bd_max_slices(max_ctx);
    const size_t n_scores = rows * FA_Q_HEADS * (size_t)max_ctx, n_stats = rows * FA_Q_HEADS * max_chunks * 2, n_part = rows * FA_Q_HEADS * max_chunks * FA_HEAD_DIM;
    return (3 * n_hidden + n_proj + 3 * n_att + n_mlp + n_logits) * sizeof(bf16) + (n_scores + n_stats + n_part) * sizeof(float) + 4096;
}

extern "C" size_t qwen35_b200_batched_scratch_bytes(int batch, int max_ctx) {
    if (batch <= 0 || max_ctx <= 0) return 0;
    return batched_scratch_total(batch, max_ctx);
}

#define Q35_TRYB(expr)                       \
    do {                                     \
        const int st__ = (expr);             \
        if (st__ != QWEN35_OK) return st__;  \
    } while (0)

extern "C" int qwen35_b200_decode_batched(const Qwen35BatchedArgs* in, qwen35_stream_t stream_) {
    using namespace q35;
    cudaStream_t stream = (cudaStream_t)stream_;
    if (!in) { set_error("null args"); return QWEN35_ERR_BAD_ARG; }
    const int B = in->batch;
    if (B <= 0 || B > 1024 || in->max_ctx <= 0 || in->max_ctx > 8192 || in->max_pages * KV_PAGE < in->max_ctx) {
        set_error("batched decode: batch %d, max_ctx %d, max_pages %d out of range (batch <= 1024, max_ctx <= 8192 <= max_pages*64)", B, in->max_ctx, in->max_pages);
        return QWEN35_ERR_BAD_ARG;
    }
    if (!in->tokens_in || !in->tokens_out || !in->positions || !in->block_table || !in->k_pages || !in->v_pages || !in->dn_states || !in->conv_bufs ||
        !in->embed_weight || !in->layer_weights || !in->fused_layer_weights || !in->lm_head_weight || !in->final_norm_weight) {
        set_error("null tensor pointer");
        return QWEN35_ERR_BAD_ARG;
    }
    // Layer tables on the host: the caller's host copies when given, else the library's copy of the device tables
    // (read back once per pair of table pointers, as for prefill)
    const LayerRec* layers_h = reinterpret_cast<const LayerRec*>(in->layer_weights_host);
    const PrefillFusedB* fused_h = reinterpret_cast<const PrefillFusedB*>(in->fused_layer_weights_host);
    HostTables tables;           // this call's own copy: a concurrent forget / eviction cannot pull it away
    if (!layers_h || !fused_h) {
        if (!in->layer_weights || !in->fused_layer_weights) { set_error("batched decode: null layer tables"); return QWEN35_ERR_BAD_ARG; }
        if (!host_layer_tables(in->layer_weights, in->fused_layer_weights, &tables)) return QWEN35_ERR_CUDA;
        layers_h = tables.layers;
        fused_h = tables.fused;
    }
    static PerDeviceOnce attr_done;
    if (attr_done.pending()) {
        Q35_CUDA_OK(cudaFuncSetAttribute(bd_att_scores_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, BD_SC_SMEM));
        Q35_CUDA_OK(cudaFuncSetAttribute(bd_att_pv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, BD_PV_SMEM));
        attr_done.mark();
    }
    // scratch rows of B tokens
    const size_t rows = (size_t)B;
    const size_t n_hidden = rows * HIDDEN, n_proj = rows * DN_PROJ_ROWS, n_att = rows * 2048, n_mlp = rows * INTER, n_logits = rows * VOCAB;
    const int max_chunks = bd_max_slices(in->max_ctx);
    const size_t n_scores = rows * FA_Q_HEADS * (size_t)in->max_ctx, n_stats = rows * FA_Q_HEADS * max_chunks * 2,
                 n_part = rows * FA_Q_HEADS * max_chunks * FA_HEAD_DIM;
    const size_t total = batched_scratch_total(B, in->max_ctx);
    char* base;
    if (in->scratch) {                       // caller-owned scratch: needed when two calls run concurrently on two streams
        if (in->scratch_bytes < total || ((uintptr_t)in->scratch & 255)) {
            set_error("batched decode: scratch of %zu bytes given (256-byte aligned?), %zu needed", in->scratch_bytes, total);
            return QWEN35_ERR_BAD_ARG;
        }
        base = (char*)in->scratch;
    } else {
        base = (char*)batched_scratch(total);
        if (!base) return QWEN35_ERR_CUDA;
    }
    int* status_word = (int*)get_workspace();      // the sticky device status word qwen35_b200_status() reads (the GEMMs use it too)
    if (!status_word) return QWEN35_ERR_CUDA;
    bf16* hidden = (bf16*)base;
    bf16* resid = hidden + n_hidden;
    bf16* normed = resid + n_hidden;
    bf16* proj = normed + n_hidden;
    bf16* qbuf = proj + n_proj;
    bf16* core = qbuf + n_att;
    bf16* attn = core + n_att;
    bf16* mlp = attn + n_att;
    bf16* logits = mlp + n_mlp;
    float* att_scores = reinterpret_cast<float*>((reinterpret_cast<uintptr_t>(logits + n_logits) + 255) & ~(uintptr_t)255);
    float* att_stats = att_scores + n_scores;
    float* att_part = att_stats + n_stats;
    RopeTable rt;
    for (int i = 0; i < FA_ROT / 2; ++i) rt.f[i] = 1.0f / (float)std::pow(1.0e7, (double)((float)(2 * i) / (float)FA_ROT));
    const size_t conv_stride = (size_t)N_DN * DN_CONV_CH * 4, state_stride = (size_t)N_DN * DN_HEADS * DN_V * DN_K;
    const int n_layers = in->dbg_num_layers > 0 ? in->dbg_num_layers : NUM_LAYERS;
    const size_t page_layer_stride = (size_t)in->num_pages * FA_KV_HEADS * KV_PAGE * FA_HEAD_DIM;

    // a step is ~300 dependent launches (replayed as a CUDA graph): programmatic dependent launch lets each kernel be
    // scheduled while its predecessor drains; every kernel of the step starts with pdl_wait()
    PdlGuard pdl_guard;
    PdlEarlyGuard pdl_early;      // short kernels in front of every GEMM: weight tiles are under way before the inputs exist
    int i_dn = 0, i_fa = 0;
    for (int layer = 0; layer < n_layers; ++layer) {
        const LayerRec& L = layers_h[layer];
        const PrefillFusedB& F = fused_h[layer];
        if (layer > 0 && in->dbg_teacher)
            Q35_CUDA_OK(pdl_launch(bd_copy_rows_kernel, (int)((n_hidden / 8 + 255) / 256), 256, 0, stream, (const bf16*)in->dbg_teacher + (size_t)layer * n_hidden, hidden, (int)(n_hidden / 8)));
        Q35_CUDA_OK(pdl_launch(pf_rmsnorm_kernel<true>, B, 128, 0, stream, layer == 0 ? in->tokens_in : nullptr, (const bf16*)in->embed_weight, hidden, (const bf16*)L.p[0],
                                                 layer == 0 ? hidden : nullptr, normed, B, (uint8_t*)nullptr, (uint8_t*)nullptr));
        const bf16 *w_out, *w_post, *w_down;
        if (L.type == 0) {
            const int ldp = DN_PROJ_ROWS;
            Q35_TRYB(gemm_bf16(normed, HIDDEN, (const bf16*)F.proj_weight, DN_PROJ_ROWS, proj, ldp, nullptr, 0, B, DN_PROJ_ROWS, HIDDEN, 0, 0, stream));
            float* conv = (float*)in->conv_bufs + (size_t)i_dn * DN_CONV_CH * 4;
            float* state = (float*)in->dn_states + (size_t)i_dn * DN_HEADS * DN_V * DN_K;
            Q35_CUDA_OK(pdl_launch(bd_dn_step_kernel, dim3(B, DN_HEADS, DN_V / BD_DN_ROWS), 256, 0, stream, proj, ldp, (const bf16*)L.p[DN_CONV], (const bf16*)L.p[DN_ALOG],
                                                                                  (const bf16*)L.p[DN_DTBIAS], conv, conv_stride, state, state_stride, core));
            Q35_CUDA_OK(pdl_launch(bd_conv_shift_kernel, (B * DN_CONV_CH + 255) / 256, 256, 0, stream, proj, ldp, conv, conv_stride, B));
            Q35_CUDA_OK(pdl_launch(pf_gated_norm_kernel<true>, (B * DN_HEADS + 15) / 16, 256, 0, stream, core, proj, ldp, (const bf16*)L.p[DN_NORM], attn, B));
            g_launches.fetch_add(3);
            w_out = (const bf16*)L.p[DN_OUT]; w_post = (const bf16*)L.p[DN_POST_NORM]; w_down = (const bf16*)L.p[DN_DOWN];
            ++i_dn;
        } else {
            const int ldp = FA_PROJ_ROWS;
            Q35_TRYB(gemm_bf16(normed, HIDDEN, (const bf16*)F.proj_weight, FA_PROJ_ROWS, proj, ldp, nullptr, 0, B, FA_PROJ_ROWS, HIDDEN, 0, 0, stream));
            bf16* kp = (bf16*)in->k_pages + (size_t)i_fa * page_layer_stride;
            bf16* vp = (bf16*)in->v_pages + (size_t)i_fa * page_layer_stride;
            Q35_CUDA_OK(pdl_launch(bd_qk_norm_rope_kernel, (B * 12 + 7) / 8, 256, 0, stream, proj, ldp, (const bf16*)L.p[FA_QNORM], (const bf16*)L.p[FA_KNORM], rt,
                                                                         in->positions, in->block_table, in->max_pages, qbuf, kp, vp, B, in->max_ctx, status_word));
            // slices per (sequence, kv head): as many as keep the grid within the CTAs the GPU holds at once (two or three per SM)
            int n_slices = (148 * 2) / (B * FA_KV_HEADS);
            const int min_slices = ((in->max_ctx + KV_PAGE - 1) / KV_PAGE + BD_MAX_PAGES_SLICE - 1) / BD_MAX_PAGES_SLICE;   // page ids per slice are bounded
            n_slices = n_slices < min_slices ? min_slices : n_slices;
            n_slices = n_slices > max_chunks ? max_chunks : n_slices;
            const dim3 agrid(B, FA_KV_HEADS, n_slices);
            CUtensorMap tmK, tmV;
            const int pool_rows = in->num_pages * FA_KV_HEADS * KV_PAGE;
            if (!make_tmap(&tmK, kp, pool_rows, FA_HEAD_DIM, FA_HEAD_DIM, KV_PAGE) || !make_tmap(&tmV, vp, pool_rows, FA_HEAD_DIM, FA_HEAD_DIM, KV_PAGE)) {
                set_error("batched decode: tensor map of the K / V page pool failed (pool %p / %p must be 16-byte aligned)", (const void*)kp, (const void*)vp);
                return QWEN35_ERR_CUDA;
            }
            Q35_CUDA_OK(pdl_launch(bd_att_scores_kernel, agrid, 128, BD_SC_SMEM, stream, tmK, (const bf16*)qbuf, in->positions, in->block_table, in->max_pages, att_scores, att_stats, in->max_ctx, max_chunks, status_word));
            Q35_CUDA_OK(pdl_launch(bd_att_pv_kernel, agrid, 128, BD_PV_SMEM, stream, tmV, in->positions, in->block_table, in->max_pages, (const float*)att_scores, (const float*)att_stats, att_part, in->max_ctx, max_chunks, status_word));
            Q35_CUDA_OK(pdl_launch(bd_att_merge_kernel, (B * FA_Q_HEADS + 7) / 8, 256, 0, stream, att_part, in->positions, proj, ldp, attn, B, max_chunks, n_slices, in->max_ctx));
            g_launches.fetch_add(4);
            w_out = (const bf16*)L.p[FA_O]; w_post = (const bf16*)L.p[FA_POST_NORM]; w_down = (const bf16*)L.p[FA_DOWN];
            ++i_fa;
        }
        Q35_TRYB(gemm_bf16(attn, 2048, w_out, HIDDEN, resid, HIDDEN, hidden, HIDDEN, B, HIDDEN, 2048, 1, 0, stream));
        Q35_CUDA_OK(pdl_launch(pf_rmsnorm_kernel<true>, B, 128, 0, stream, nullptr, nullptr, resid, w_post, nullptr, normed, B, (uint8_t*)nullptr, (uint8_t*)nullptr));
        Q35_TRYB(gemm_bf16(normed, HIDDEN, (const bf16*)F.gate_up_weight, 2 * INTER, mlp, INTER, nullptr, 0, B, INTER, HIDDEN, 2, INTER, stream));
        Q35_TRYB(gemm_bf16(mlp, INTER, w_down, HIDDEN, hidden, HIDDEN, resid, HIDDEN, B, HIDDEN, INTER, 1, 0, stream));
        g_launches.fetch_add(2);
        if (in->dbg_hidden)
            Q35_CUDA_OK(pdl_launch(bd_copy_rows_kernel, (int)((n_hidden / 8 + 255) / 256), 256, 0, stream, hidden, (bf16*)in->dbg_hidden + (size_t)layer * n_hidden, (int)(n_hidden / 8)));
    }
    Q35_CUDA_OK(pdl_launch(pf_rmsnorm_kernel<true>, B, 128, 0, stream, nullptr, nullptr, hidden, (const bf16*)in->final_norm_weight, nullptr, normed, B, (uint8_t*)nullptr, (uint8_t*)nullptr));
    Q35_TRYB(gemm_bf16(normed, HIDDEN, (const bf16*)in->lm_head_weight, VOCAB, logits, VOCAB, nullptr, 0, B, VOCAB, HIDDEN, 0, 0, stream));
    Q35_CUDA_OK(pdl_launch(bd_argmax_kernel, B, 1024, 0, stream, logits, in->tokens_out, in->advance_positions ? in->positions : nullptr, in->max_ctx));
    if (in->logits_out) Q35_CUDA_OK(cudaMemcpyAsync(in->logits_out, logits, n_logits * sizeof(bf16), cudaMemcpyDeviceToDevice, stream));
    g_launches.fetch_add(2);
    Q35_CUDA_OK(cudaGetLastError());
    return QWEN35_OK;
}
