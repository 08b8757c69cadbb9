// Tree verification for the 27B-class hybrid target: one forward pass over the N nodes of a draft tree (DFS order,
// node 0 = root) on top of a committed context, then the accepted-path walk and the commit of that path's state.
// Replaces the ggml graph of the reference's target (models/qwen35_27b/src/qwen35_target_graph.cpp:281-804) and the
// host-side tree code around it (models/qwen35_27b/test/test_dflash.cpp:396-442, 1355-1521).
//
// A node's result is that of the sequential model run on its root-to-node token path:
//   full attention   K/V of node t go to cache slot past + t; node t sees slots < past and its ancestors-or-self
//                    (a 64-bit ancestor word per node is the tree mask); position = past + depth(t)
//   DeltaNet         the short conv gathers each node's three predecessors along its parent chain (then the
//                    committed conv state); the recurrence runs in DFS order, reloads the parent's state when the
//                    DFS order branches, and persists every node's post-state as f16 for the commit
// Weights are Q4_K super-blocks (256 weights in 144 bytes).  A linear layer is one launch of the tcgen05 split-K
// GEMM whose weight operand is dequantised by the kernel itself into the swizzled shared-memory tile (HBM sees the
// 4.5-bit weights once, bf16 weights never exist in global memory); the attention products run on mma.sync tiles
// with K/V staged through shared memory.
// Dimensions are run-time values (head_dim 256 and DeltaNet head size 128 are fixed).
#include <cuda_fp16.h>

#include <cmath>

#include "common.cuh"
#include "norm_kernels.cuh"
#include "runtime.h"

namespace q35 {

int gemm_bf16(const bf16* A, int lda, const bf16* B, int b_rows, bf16* C, int ldc, const bf16* R, int ldr,
              int M, int N, int K, int epi, int up_row_offset, cudaStream_t stream);
int gemm_q4k(const bf16* A, int lda, const uint8_t* W, int w_rows, bf16* C, int ldc, const bf16* R, int ldr,
             int M, int N, int K, int epi, int up_row_offset, cudaStream_t stream);

constexpr int TV_MAX_NODES = 40;       // query rows of one kv head (nodes x q-per-kv) must fit shared memory
constexpr int TV_HD = 256;             // attention head size
constexpr int TV_DN = 128;             // DeltaNet head size
constexpr int TV_CHUNK = 128;          // keys per attention CTA
constexpr int TV_QSTRIDE = TV_HD + 8;  // padded shared-memory row (bf16 elements): conflict-free fragment loads
constexpr int TV_PSTRIDE = TV_CHUNK + 8;

struct TvDims {
    int n_layers, hidden, ffn, vocab, q_heads, kv_heads, head_dim, dn_k_heads, dn_v_heads, dn_dim, rot_dim, fa_period;
    float theta, eps;
};

// ------------------------------------------------ Q4_K ------------------------------------------------
// super-block: f16 d, f16 dmin, 12 bytes of 6-bit scales and mins for 8 sub-blocks of 32, 128 bytes of nibbles.
// value = (d * sc) * q - (dmin * m), every operation a separate f32 rounding (the published dequantisation).
__device__ __forceinline__ void q4k_scale_min(const uint8_t* s, int j, int& sc, int& m) {
    if (j < 4) { sc = s[j] & 63; m = s[j + 4] & 63; }
    else { sc = (s[j + 4] & 0xF) | ((s[j - 4] >> 6) << 4); m = (s[j + 4] >> 4) | ((s[j] >> 6) << 4); }
}

// one warp per super-block; lane l owns nibble bytes [4l, 4l+4): 4 low-nibble and 4 high-nibble weights
__device__ __forceinline__ void q4k_dequant_lane(const uint8_t* blk, int lane, float (&lo)[4], float (&hi)[4], int& e_lo) {
    const float d = __half2float(*reinterpret_cast<const __half*>(blk));
    const float dmin = __half2float(*reinterpret_cast<const __half*>(blk + 2));
    const int g = lane >> 3, pos = (lane & 7) * 4;
    int sc0, m0, sc1, m1;
    q4k_scale_min(blk + 4, 2 * g, sc0, m0);
    q4k_scale_min(blk + 4, 2 * g + 1, sc1, m1);
    const float d0 = __fmul_rn(d, (float)sc0), mm0 = __fmul_rn(dmin, (float)m0);
    const float d1 = __fmul_rn(d, (float)sc1), mm1 = __fmul_rn(dmin, (float)m1);
    const uint32_t qb = *reinterpret_cast<const uint32_t*>(blk + 16 + lane * 4);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint32_t b = (qb >> (8 * i)) & 0xFF;
        lo[i] = __fsub_rn(__fmul_rn(d0, (float)(b & 0xF)), mm0);
        hi[i] = __fsub_rn(__fmul_rn(d1, (float)(b >> 4)), mm1);
    }
    e_lo = g * 64 + pos;          // low-nibble weights at e_lo.., high-nibble weights at e_lo + 32..
}

// rows [row0, row0+rows) of a [*, cols] matrix -> bf16 panel (and / or f32 copy)
__global__ void __launch_bounds__(256) tv_dequant_q4k_kernel(const uint8_t* __restrict__ blocks, size_t first_block, size_t n_blocks,
                                                             bf16* __restrict__ out_bf16, float* __restrict__ out_f32) {
    const size_t b = (size_t)blockIdx.x * 8 + (threadIdx.x >> 5);
    if (b >= n_blocks) return;
    const int lane = threadIdx.x & 31;
    float lo[4], hi[4];
    int e;
    q4k_dequant_lane(blocks + (first_block + b) * 144, lane, lo, hi, e);
    if (out_bf16) {
        bf16* o = out_bf16 + b * 256 + e;
        const __nv_bfloat162 l0 = __halves2bfloat162(f2bf(lo[0]), f2bf(lo[1])), l1 = __halves2bfloat162(f2bf(lo[2]), f2bf(lo[3]));
        const __nv_bfloat162 h0 = __halves2bfloat162(f2bf(hi[0]), f2bf(hi[1])), h1 = __halves2bfloat162(f2bf(hi[2]), f2bf(hi[3]));
        *reinterpret_cast<uint2*>(o) = make_uint2(*reinterpret_cast<const uint32_t*>(&l0), *reinterpret_cast<const uint32_t*>(&l1));
        *reinterpret_cast<uint2*>(o + 32) = make_uint2(*reinterpret_cast<const uint32_t*>(&h0), *reinterpret_cast<const uint32_t*>(&h1));
    }
    if (out_f32) {
        float* o = out_f32 + b * 256 + e;
        *reinterpret_cast<float4*>(o) = make_float4(lo[0], lo[1], lo[2], lo[3]);
        *reinterpret_cast<float4*>(o + 32) = make_float4(hi[0], hi[1], hi[2], hi[3]);
    }
}

// embedding rows of the node tokens, bf16
__global__ void __launch_bounds__(32) tv_embed_q4k_kernel(const uint8_t* __restrict__ embd, const int* __restrict__ tokens, int hidden,
                                                          bf16* __restrict__ out) {
    pdl_wait();
    const int t = blockIdx.x, blk = blockIdx.y, lane = threadIdx.x;
    const size_t b = (size_t)tokens[t] * (hidden / 256) + blk;
    float lo[4], hi[4];
    int e;
    q4k_dequant_lane(embd + b * 144, lane, lo, hi, e);
    bf16* o = out + (size_t)t * hidden + blk * 256 + e;
#pragma unroll
    for (int i = 0; i < 4; ++i) { o[i] = f2bf(lo[i]); o[32 + i] = f2bf(hi[i]); }
}

// ------------------------------------------- tree bookkeeping -------------------------------------------
// depth[t] and the ancestor-or-self word anc[t] (bit j set: node j is on the root-to-t path); parents[t] < t.
// For the tree delta rule it also plans where each node's starting state comes from and which post-states a CTA keeps
// in one of its TV_DN_SLOTS shared-memory slots:
//   src[t]  = -2 continue from node t-1's registers; -1 read from memory (the parent's persisted state, or the
//             committed state for a root); s >= 0 read the parent's state from slot s
//   save[t] = slot that keeps node t's post-state for a later child that is not t+1, or -1
// A slot is held from its node until that node's last such child; when none is free the child reads from memory.
constexpr int TV_DN_SLOTS = 8;
__global__ void tv_tree_prep_kernel(const int* __restrict__ parents, int n, int* __restrict__ depth, unsigned long long* __restrict__ anc,
                                    int* __restrict__ src, int* __restrict__ save) {
    pdl_wait();
    if (threadIdx.x != 0 || blockIdx.x != 0) return;
    int last[TV_MAX_NODES], owner[TV_DN_SLOTS];
    for (int t = 0; t < n; ++t) {
        const int p = parents[t];
        const bool ok = p >= 0 && p < t;
        depth[t] = ok ? depth[p] + 1 : 0;
        anc[t] = (ok ? anc[p] : 0ull) | (1ull << t);
        last[t] = -1;
    }
    for (int c = 1; c < n; ++c) {
        const int p = parents[c];
        if (p >= 0 && p < c && p != c - 1) last[p] = c;
    }
    for (int i = 0; i < TV_DN_SLOTS; ++i) owner[i] = -1;
    for (int t = 0; t < n; ++t) {
        const int p = parents[t];
        int from = -1;
        if (t > 0 && p == t - 1) from = -2;
        else if (p >= 0 && p < t)
            for (int i = 0; i < TV_DN_SLOTS; ++i) if (owner[i] == p) from = i;
        src[t] = from;
        for (int i = 0; i < TV_DN_SLOTS; ++i) if (owner[i] >= 0 && last[owner[i]] <= t) owner[i] = -1;
        int keep = -1;
        if (last[t] > t)
            for (int i = 0; i < TV_DN_SLOTS && keep < 0; ++i) if (owner[i] < 0) { owner[i] = t; keep = i; }
        save[t] = keep;
    }
}

// K / V cache rows, by kv_type (the reference's cache types, qwen35_target_graph.cpp:110-122, plus this library's bf16):
//   0 bf16 [256] (512 bytes);
//   1 Q8_0 (the reference's default): 8 blocks of {f16 d, 32 x int8} = 272 bytes, d = amax / 127, q = roundf(x / d);
//   2 Q4_0: 8 blocks of {f16 d, 16 bytes of nibbles} = 144 bytes, d = (the element of largest magnitude) / -8,
//     q = min(15, trunc(x / d + 8.5)), byte j = q[j] | q[j + 16] << 4, value d (q - 8);
//   3 F16 [256] (512 bytes).
// Quantised from the f32 values when a row is written and read back as the bf16 operand bf16(value).
constexpr int TV_KV_BF16 = 0, TV_KV_Q8_0 = 1, TV_KV_Q4_0 = 2, TV_KV_F16 = 3;
constexpr int TV_Q8_ROW = (TV_HD / 32) * 34;
constexpr int TV_Q4_ROW = (TV_HD / 32) * 18;
constexpr int TV_PV_THREADS = 512;      // scores and P.V kernels: 16 warps share a chunk (latency-bound with 8; P.V: 99 exp + divide per thread)
__host__ __device__ constexpr int tv_kv_row_bytes(int kv_type) { return kv_type == TV_KV_Q8_0 ? TV_Q8_ROW : kv_type == TV_KV_Q4_0 ? TV_Q4_ROW : TV_HD * 2; }
// bytes of the raw staging buffer the attention kernels need beside the bf16 tile (the 512-byte row types land in the tile)
__host__ __device__ constexpr int tv_kv_raw_bytes(int kv_type) { return kv_type == TV_KV_Q8_0 ? TV_CHUNK * TV_Q8_ROW : kv_type == TV_KV_Q4_0 ? TV_CHUNK * TV_Q4_ROW : 0; }

// one warp = one 32-element block: lane holds element `lane` of the block
__device__ __forceinline__ void tv_q8_store_block(unsigned char* blk, float v, int lane) {
    const float amax = warp_max(fabsf(v));
    const float d = amax / 127.0f;
    const float id = d != 0.f ? 1.0f / d : 0.f;
    blk[2 + lane] = (unsigned char)(signed char)(int)roundf(v * id);
    if (lane == 0) *reinterpret_cast<__half*>(blk) = __float2half_rn(d);
}
__device__ __forceinline__ void tv_q4_store_block(unsigned char* blk, float v, int lane) {
    // the element of largest magnitude, the first one among equals, with its sign
    float best = fabsf(v);
    int bi = lane;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ob = __shfl_xor_sync(0xffffffffu, best, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ob > best || (ob == best && oi < bi)) { best = ob; bi = oi; }
    }
    const float mx = __shfl_sync(0xffffffffu, v, bi);
    const float d = mx * -0.125f;
    const float id = d != 0.f ? __fdiv_rn(1.0f, d) : 0.f;
    const int q = min(15, (int)__fadd_rn(__fmul_rn(v, id), 8.5f));        // >= 0.5 before truncation; no fused multiply-add
    const int hi = __shfl_down_sync(0xffffffffu, q, 16);
    if (lane < 16) blk[2 + lane] = (unsigned char)(q | (hi << 4));
    if (lane == 0) *reinterpret_cast<__half*>(blk) = __float2half_rn(d);
}
// 128 threads write one cache row from its 256 f32 values: thread tid holds elements tid and tid + 128
__device__ __forceinline__ void tv_store_kv_row(unsigned char* row, float a, float b, int tid, int kv_type) {
    if (kv_type == TV_KV_Q8_0) {                                   // warp w holds blocks w and 4 + w
        tv_q8_store_block(row + (tid >> 5) * 34, a, tid & 31);
        tv_q8_store_block(row + (4 + (tid >> 5)) * 34, b, tid & 31);
    } else if (kv_type == TV_KV_Q4_0) {
        tv_q4_store_block(row + (tid >> 5) * 18, a, tid & 31);
        tv_q4_store_block(row + (4 + (tid >> 5)) * 18, b, tid & 31);
    } else if (kv_type == TV_KV_F16) {
        __half* dst = reinterpret_cast<__half*>(row);
        dst[tid] = __float2half_rn(a); dst[tid + 128] = __float2half_rn(b);
    } else {
        bf16* dst = reinterpret_cast<bf16*>(row);
        dst[tid] = f2bf(a); dst[tid + 128] = f2bf(b);
    }
}

// stage 128 cache rows [j0, j0 + 128) of one kv head into the padded bf16 tile; rows >= L are zero.  512-byte rows are copied
// straight into the tile (F16 rows are converted in place afterwards); Q8_0 and Q4_0 rows are copied raw into `raw`;
// tv_finish_rows converts after the copies landed.
template <int KT>
__device__ __forceinline__ void tv_stage_rows(bf16* tile, unsigned char* raw, const unsigned char* head_base, int j0, int L, int tid, int nthr = 256) {
    if (KT == TV_KV_Q8_0 || KT == TV_KV_Q4_0) {
        constexpr int ROW = tv_kv_row_bytes(KT);
        for (int i = tid; i < TV_CHUNK * (ROW / 16); i += nthr) {
            const int k = i / (ROW / 16), c = i % (ROW / 16);
            if (j0 + k < L) cp_async16(raw + (size_t)k * ROW + c * 16, head_base + (size_t)(j0 + k) * ROW + c * 16);
        }
    } else {
        for (int i = tid; i < TV_CHUNK * (TV_HD / 8); i += nthr) {
            const int k = i / (TV_HD / 8), c8 = i % (TV_HD / 8);
            bf16* dst = tile + (size_t)k * TV_QSTRIDE + c8 * 8;
            if (j0 + k < L) cp_async16(dst, head_base + ((size_t)(j0 + k) * TV_HD + c8 * 8) * 2);
            else *reinterpret_cast<uint4*>(dst) = make_uint4(0, 0, 0, 0);
        }
    }
}
// call after cp_async_wait_all() + __syncthreads(); converts the rows of the other types to bf16 and synchronises again
template <int KT>
__device__ __forceinline__ void tv_finish_rows(bf16* tile, const unsigned char* raw, int j0, int L, int tid, int nthr = 256) {
    if (KT == TV_KV_BF16) return;
    if (KT == TV_KV_F16) {
        for (int i = tid; i < TV_CHUNK * (TV_HD / 8); i += nthr) {
            const int k = i / (TV_HD / 8), c8 = i % (TV_HD / 8);
            if (j0 + k >= L) continue;                                    // zero rows stay zero
            uint4* p = reinterpret_cast<uint4*>(tile + (size_t)k * TV_QSTRIDE + c8 * 8);
            const uint4 h = *p;
            const uint32_t in[4] = {h.x, h.y, h.z, h.w};
            uint32_t o[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&in[e]));
                const __nv_bfloat162 pr = __floats2bfloat162_rn(f.x, f.y);
                o[e] = *reinterpret_cast<const uint32_t*>(&pr);
            }
            *p = make_uint4(o[0], o[1], o[2], o[3]);
        }
        __syncthreads();
        return;
    }
    for (int i = tid; i < TV_CHUNK * (TV_HD / 32); i += nthr) {
        const int k = i / (TV_HD / 32), b = i % (TV_HD / 32);
        uint32_t o[16];
        if (j0 + k >= L) {
#pragma unroll
            for (int e = 0; e < 16; ++e) o[e] = 0u;
        } else if (KT == TV_KV_Q8_0) {
            const unsigned char* blk = raw + (size_t)k * TV_Q8_ROW + b * 34;
            const float d = __half2float(*reinterpret_cast<const __half*>(blk));
#pragma unroll
            for (int e = 0; e < 16; ++e) {
                const unsigned short two = *reinterpret_cast<const unsigned short*>(blk + 2 + 2 * e);
                const __nv_bfloat162 pr = __floats2bfloat162_rn(d * (float)(signed char)(two & 0xFF), d * (float)(signed char)(two >> 8));
                o[e] = *reinterpret_cast<const uint32_t*>(&pr);
            }
        } else {
            // Q4_0: byte j holds elements j (low nibble) and j + 16 (high nibble); output pair e = elements 2 e, 2 e + 1
            const unsigned char* blk = raw + (size_t)k * TV_Q4_ROW + b * 18;
            const float d = __half2float(*reinterpret_cast<const __half*>(blk));
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                const unsigned short two = *reinterpret_cast<const unsigned short*>(blk + 2 + 2 * e);     // bytes 2 e, 2 e + 1
                const int b0 = two & 0xFF, b1 = two >> 8;
                const __nv_bfloat162 lo = __floats2bfloat162_rn(d * (float)((b0 & 15) - 8), d * (float)((b1 & 15) - 8));
                const __nv_bfloat162 hi = __floats2bfloat162_rn(d * (float)((b0 >> 4) - 8), d * (float)((b1 >> 4) - 8));
                o[e] = *reinterpret_cast<const uint32_t*>(&lo);
                o[8 + e] = *reinterpret_cast<const uint32_t*>(&hi);
            }
        }
        uint4* dst = reinterpret_cast<uint4*>(tile + (size_t)k * TV_QSTRIDE + b * 32);
#pragma unroll
        for (int e = 0; e < 4; ++e) dst[e] = make_uint4(o[4 * e], o[4 * e + 1], o[4 * e + 2], o[4 * e + 3]);
    }
    __syncthreads();
}

// ------------------------------------------ full attention ------------------------------------------
// one CTA (128 threads, 2 elements each) per (node, slot): q heads, then k heads, then v heads of the projection row
// [per q head: q(256) | gate(256)] [k heads] [v heads].  Head RMSNorm (plain weight), rotate-half RoPE over rot_dim.
__global__ void __launch_bounds__(128) tv_fa_prep_kernel(const bf16* __restrict__ proj, int ldp, const float* __restrict__ qn, const float* __restrict__ kn,
                                                         const int* __restrict__ depth, TvDims D, int past, int max_ctx,
                                                         bf16* __restrict__ qbuf, unsigned char* __restrict__ k_cache, unsigned char* __restrict__ v_cache, int kv_type) {
    pdl_wait();
    __shared__ float red[4];
    __shared__ float xs[TV_HD];
    const int t = blockIdx.x, slot = blockIdx.y, tid = threadIdx.x;
    const bf16* row = proj + (size_t)t * ldp;
    const int qcols = 2 * D.q_heads * TV_HD;
    if (slot >= D.q_heads + D.kv_heads) {                      // v head: copy into the cache slot
        const int kvh = slot - D.q_heads - D.kv_heads;
        const bf16* src = row + qcols + (D.kv_heads + kvh) * TV_HD;
        unsigned char* vrow = v_cache + ((size_t)kvh * max_ctx + past + t) * tv_kv_row_bytes(kv_type);
        tv_store_kv_row(vrow, bf2f(src[tid]), bf2f(src[tid + 128]), tid, kv_type);
        return;
    }
    const bool isq = slot < D.q_heads;
    const bf16* src = isq ? row + (size_t)slot * 2 * TV_HD : row + qcols + (slot - D.q_heads) * TV_HD;
    const float* w = isq ? qn : kn;
    const float a = bf2f(src[tid]), b = bf2f(src[tid + 128]);
    const float inv = rsqrt_ieee(tv_block_sum(fmaf(a, a, b * b), red) / (float)TV_HD + D.eps);
    xs[tid] = a * inv * w[tid];
    xs[tid + 128] = b * inv * w[tid + 128];
    __syncthreads();
    const float pos = (float)(past + depth[t]);
    const int half = D.rot_dim / 2;
    float y[2];
#pragma unroll
    for (int k = 0; k < 2; ++k) {
        const int e = tid + 128 * k;
        float v = xs[e];
        if (e < D.rot_dim) {
            const int i = e < half ? e : e - half;
            const float inv_freq = powf(D.theta, -(float)(2 * i) / (float)D.rot_dim);
            float sn, cs;
            sincosf(pos * inv_freq, &sn, &cs);
            v = e < half ? xs[e] * cs - xs[e + half] * sn : xs[e] * cs + xs[e - half] * sn;
        }
        y[k] = v;
    }
    if (!isq) {
        tv_store_kv_row(k_cache + ((size_t)(slot - D.q_heads) * max_ctx + past + t) * tv_kv_row_bytes(kv_type), y[0], y[1], tid, kv_type);
        return;
    }
    bf16* dst = qbuf + ((size_t)t * D.q_heads + slot) * TV_HD;
    dst[tid] = f2bf(y[0]); dst[tid + 128] = f2bf(y[1]);
}

// scores of all query rows of one kv head (row r = node * gqa + q-in-group) against one chunk of keys:
// s = (q . k) / 16 in f32, masked to -inf outside [0, past) and the node's ancestors.  grid (chunks, kv_heads).
template <int KT>
__global__ void __launch_bounds__(TV_PV_THREADS, 1) tv_att_scores_kernel(const bf16* __restrict__ qbuf, const unsigned char* __restrict__ k_cache,
                                                               const unsigned long long* __restrict__ anc, TvDims D, int n_nodes, int past,
                                                               int max_ctx, int lpad, float* __restrict__ scores) {
    pdl_wait();
    extern __shared__ __align__(16) unsigned char tv_smem[];
    bf16* Qs = reinterpret_cast<bf16*>(tv_smem);
    const int gqa = D.q_heads / D.kv_heads, R = n_nodes * gqa, mt_n = (R + 15) / 16;
    bf16* Ks = Qs + (size_t)mt_n * 16 * TV_QSTRIDE;
    const int chunk = blockIdx.x, kvh = blockIdx.y, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int j0 = chunk * TV_CHUNK, L = past + n_nodes;
    // Q rows and the K chunk go to shared memory by cp.async: every copy of the tile is in flight at once
    for (int i = tid; i < mt_n * 16 * (TV_HD / 8); i += TV_PV_THREADS) {
        const int r = i / (TV_HD / 8), c8 = i % (TV_HD / 8);
        bf16* dst = Qs + (size_t)r * TV_QSTRIDE + c8 * 8;
        if (r < R) cp_async16(dst, qbuf + ((size_t)(r / gqa) * D.q_heads + kvh * gqa + r % gqa) * TV_HD + c8 * 8);
        else *reinterpret_cast<uint4*>(dst) = make_uint4(0, 0, 0, 0);
    }
    unsigned char* raw = reinterpret_cast<unsigned char*>(Ks + (size_t)TV_CHUNK * TV_QSTRIDE);      // the quantised types only
    tv_stage_rows<KT>(Ks, raw, k_cache + (size_t)kvh * max_ctx * tv_kv_row_bytes(KT), j0, L, tid, TV_PV_THREADS);
    cp_async_wait_all();
    __syncthreads();
    tv_finish_rows<KT>(Ks, raw, j0, L, tid, TV_PV_THREADS);
    const int g = lane >> 2, c = lane & 3;
    // 16 warps: warp w owns the 16 keys [16 kp, 16 kp + 16), kp = w mod 8, of the chunk = two 8-key MMA tiles (their K
    // fragments, by ldmatrix, stay in registers for the whole kernel) and every other pair of query tiles (w / 8).  Query
    // tiles go two at a time, so four independent accumulator chains are in flight (one chain of 16 dependent MMAs at a
    // time left the tensor pipe waiting on its own latency).
    static_assert(TV_CHUNK / 16 == 8 && TV_PV_THREADS == 512, "8 key pairs x 2 query-tile phases = 16 warps");
    const int kp = warp & 7;
    uint32_t bfr[TV_HD / 16][4];
#pragma unroll
    for (int s = 0; s < TV_HD / 16; ++s)
        ldsm_x4(bfr[s], Ks + (size_t)(kp * 16 + (lane & 7) + 8 * (lane >> 4)) * TV_QSTRIDE + s * 16 + 8 * ((lane >> 3) & 1));
    auto emit = [&](const float (&acc)[4], int mt, int nt) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int r = mt * 16 + g + 8 * h;
            if (r >= R) continue;
            const unsigned long long am = anc[r / gqa];
            float* dst = scores + ((size_t)kvh * R + r) * lpad + j0 + nt * 8 + 2 * c;
            float2 out;
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                const int j = j0 + nt * 8 + 2 * c + e;
                const bool vis = j < past || (j < L && ((am >> (j - past)) & 1ull));
                (e ? out.y : out.x) = vis ? acc[2 * h + e] * 0.0625f : -INFINITY;
            }
            *reinterpret_cast<float2*>(dst) = out;
        }
    };
    for (int mt = 2 * (warp >> 3); mt < mt_n; mt += 4) {
        const bool two = mt + 1 < mt_n;                       // warp-uniform
        float acc00[4] = {0.f, 0.f, 0.f, 0.f}, acc01[4] = {0.f, 0.f, 0.f, 0.f}, acc10[4] = {0.f, 0.f, 0.f, 0.f}, acc11[4] = {0.f, 0.f, 0.f, 0.f};
        const bf16* qa = Qs + (size_t)(mt * 16 + (lane & 15)) * TV_QSTRIDE + (lane >> 4) * 8;
        const bf16* qb = qa + (two ? 16 * TV_QSTRIDE : 0);
#pragma unroll
        for (int s = 0; s < TV_HD / 16; ++s) {
            uint32_t a0[4], a1[4];
            ldsm_x4(a0, qa + s * 16);
            ldsm_x4(a1, qb + s * 16);
            mma_16816(acc00, a0, bfr[s][0], bfr[s][1]);
            mma_16816(acc01, a0, bfr[s][2], bfr[s][3]);
            mma_16816(acc10, a1, bfr[s][0], bfr[s][1]);
            mma_16816(acc11, a1, bfr[s][2], bfr[s][3]);
        }
        emit(acc00, mt, 2 * kp); emit(acc01, mt, 2 * kp + 1);
        if (two) { emit(acc10, mt + 1, 2 * kp); emit(acc11, mt + 1, 2 * kp + 1); }
    }
}

// softmax statistics of every query row over the whole (masked) key range: one warp per row
__global__ void __launch_bounds__(256) tv_att_stats_kernel(const float* __restrict__ scores, int rows, int lpad, int len, float* __restrict__ stats) {
    pdl_wait();
    const int r = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (r >= rows) return;
    const float* s = scores + (size_t)r * lpad;
    // len is a multiple of the 128-key chunk: 16-byte loads, element order of the sum = (lane, then key) as before per lane
    float mx = -INFINITY;
#pragma unroll 4
    for (int j = lane * 4; j < len; j += 128) {
        const float4 v = *reinterpret_cast<const float4*>(s + j);
        mx = fmaxf(fmaxf(mx, fmaxf(v.x, v.y)), fmaxf(v.z, v.w));
    }
    mx = warp_max(mx);
    float sm = 0.f;
#pragma unroll 4
    for (int j = lane * 4; j < len; j += 128) {
        const float4 v = *reinterpret_cast<const float4*>(s + j);
        sm += expf(v.x - mx); sm += expf(v.y - mx); sm += expf(v.z - mx); sm += expf(v.w - mx);
    }
    sm = warp_sum(sm);
    if (lane == 0) { stats[2 * r] = mx; stats[2 * r + 1] = sm; }
}

// partial P.V of one chunk of keys for all query rows of one kv head; P = bf16(exp(s - m) / l).  grid (chunks, kv_heads).
// The V chunk is staged row-major by cp.async and read as the B operand with ldmatrix.trans; P goes to shared memory
// row-major and is read as the A operand with ldmatrix.
template <int KT>
__global__ void __launch_bounds__(TV_PV_THREADS, 1) tv_att_pv_kernel(const unsigned char* __restrict__ v_cache, const float* __restrict__ scores, const float* __restrict__ stats,
                                                           TvDims D, int n_nodes, int past, int max_ctx, int lpad, float* __restrict__ partial) {
    pdl_wait();
    extern __shared__ __align__(16) unsigned char tv_smem[];
    bf16* Vs = reinterpret_cast<bf16*>(tv_smem);                     // [TV_CHUNK keys][TV_QSTRIDE]
    bf16* Ps = Vs + (size_t)TV_CHUNK * TV_QSTRIDE;                   // [rows][TV_PSTRIDE keys]
    const int gqa = D.q_heads / D.kv_heads, R = n_nodes * gqa, mt_n = (R + 15) / 16;
    const int chunk = blockIdx.x, kvh = blockIdx.y, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int j0 = chunk * TV_CHUNK, L = past + n_nodes;
    unsigned char* raw = reinterpret_cast<unsigned char*>(Ps + (size_t)mt_n * 16 * TV_PSTRIDE);      // the quantised types only
    tv_stage_rows<KT>(Vs, raw, v_cache + (size_t)kvh * max_ctx * tv_kv_row_bytes(KT), j0, L, tid, TV_PV_THREADS);
    // P rows (overlapping the copies above): a warp takes one row at a time, a lane four consecutive keys, so the score
    // loads are 16-byte, coalesced and several rows deep in flight
    static_assert(TV_CHUNK == 128, "one warp covers a 128-key row with four keys per lane");
#pragma unroll 7
    for (int r = warp; r < mt_n * 16; r += TV_PV_THREADS / 32) {
        float4 sc = make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
        float m = 0.f, l = 1.f;
        if (r < R) {
            const size_t gr = (size_t)kvh * R + r;
            sc = *reinterpret_cast<const float4*>(scores + gr * lpad + j0 + lane * 4);
            m = stats[2 * gr]; l = stats[2 * gr + 1];
        }
        const float p0 = (sc.x == -INFINITY) ? 0.f : expf(sc.x - m) / l, p1 = (sc.y == -INFINITY) ? 0.f : expf(sc.y - m) / l;
        const float p2 = (sc.z == -INFINITY) ? 0.f : expf(sc.z - m) / l, p3 = (sc.w == -INFINITY) ? 0.f : expf(sc.w - m) / l;
        const __nv_bfloat162 lo = __floats2bfloat162_rn(p0, p1), hi = __floats2bfloat162_rn(p2, p3);
        *reinterpret_cast<uint2*>(Ps + (size_t)r * TV_PSTRIDE + lane * 4) = make_uint2(*reinterpret_cast<const uint32_t*>(&lo), *reinterpret_cast<const uint32_t*>(&hi));
    }
    cp_async_wait_all();
    __syncthreads();
    tv_finish_rows<KT>(Vs, raw, j0, L, tid, TV_PV_THREADS);
    const int g = lane >> 2, c = lane & 3;
    const int n_chunks = gridDim.x;
    for (int np = warp; np < TV_HD / 16; np += TV_PV_THREADS / 32) {                   // pairs of 8-dim output tiles
        uint32_t bfr[TV_CHUNK / 16][4];
#pragma unroll
        for (int s = 0; s < TV_CHUNK / 16; ++s)
            ldsm_x4_trans(bfr[s], Vs + (size_t)(s * 16 + (lane & 7) + 8 * ((lane >> 3) & 1)) * TV_QSTRIDE + np * 16 + 8 * (lane >> 4));
        for (int mt = 0; mt < mt_n; ++mt) {
            float acc0[4] = {0.f, 0.f, 0.f, 0.f}, acc1[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int s = 0; s < TV_CHUNK / 16; ++s) {
                uint32_t a[4];
                ldsm_x4(a, Ps + (size_t)(mt * 16 + (lane & 15)) * TV_PSTRIDE + s * 16 + (lane >> 4) * 8);
                mma_16816(acc0, a, bfr[s][0], bfr[s][1]);
                mma_16816(acc1, a, bfr[s][2], bfr[s][3]);
            }
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int r = mt * 16 + g + 8 * h;
                if (r < R) {
                    float* dst = partial + (((size_t)kvh * R + r) * n_chunks + chunk) * TV_HD + np * 16 + 2 * c;
                    *reinterpret_cast<float2*>(dst) = make_float2(acc0[2 * h], acc0[2 * h + 1]);
                    *reinterpret_cast<float2*>(dst + 8) = make_float2(acc1[2 * h], acc1[2 * h + 1]);
                }
            }
        }
    }
}

// sum of the chunk partials in chunk order, times sigmoid(gate), one rounding to bf16.  grid (nodes, q_heads), 128 threads
__global__ void __launch_bounds__(128) tv_att_merge_kernel(const float* __restrict__ partial, const bf16* __restrict__ proj, int ldp, TvDims D,
                                                           int n_nodes, int n_chunks, bf16* __restrict__ out) {
    pdl_trigger();      // the projection GEMM that follows loads and dequantises its first weights beside this kernel
    pdl_wait();
    const int t = blockIdx.x, hq = blockIdx.y, tid = threadIdx.x;
    const int gqa = D.q_heads / D.kv_heads, R = n_nodes * gqa, kvh = hq / gqa, r = t * gqa + hq % gqa;
    const float* pb = partial + ((size_t)kvh * R + r) * n_chunks * TV_HD;
    float a0 = 0.f, a1 = 0.f;
    for (int ch = 0; ch < n_chunks; ++ch) {
        const float2 v = *reinterpret_cast<const float2*>(pb + (size_t)ch * TV_HD + 2 * tid);
        a0 += v.x; a1 += v.y;
    }
    const bf16* gate = proj + (size_t)t * ldp + (size_t)hq * 2 * TV_HD + TV_HD + 2 * tid;
    bf16* o = out + ((size_t)t * D.q_heads + hq) * TV_HD + 2 * tid;
    o[0] = f2bf(a0 * sigmoid_f(bf2f(gate[0])));
    o[1] = f2bf(a1 * sigmoid_f(bf2f(gate[1])));
}

// --------------------------------------------- DeltaNet ---------------------------------------------
// tree short-conv + SiLU, then what the delta rule needs of it, in one kernel.  grid (nodes, conv channels / 128),
// 128 threads: a block is one head-sized slice of the conv channels.
//   conv: taps of node t = its three predecessors on the parent chain, continuing into the committed conv state
//         [3][channels] (row 2 newest) when the chain ends (qwen35_target_graph.cpp:462-496); the raw projection row of
//         every node is kept for the commit
//   q and k slices: L2 norm of the head (q also scaled by 1/sqrt(128))
//   v slice of head h: beta = sigmoid(b), decay = exp(softplus(a + dt_bias) * ssm_a) for (node, h)
__global__ void __launch_bounds__(128) tv_dn_conv_norm_kernel(const bf16* __restrict__ proj, int ldp, const int* __restrict__ parents,
                                                              const float* __restrict__ conv_state, const float* __restrict__ conv_w, int conv_ch,
                                                              const bf16* __restrict__ ba, int ldba, const float* __restrict__ ssm_a,
                                                              const float* __restrict__ dt_bias, TvDims D, float* __restrict__ qkv,
                                                              float* __restrict__ node_conv, float* __restrict__ gate /* [nodes][v_heads][2] */) {
    pdl_wait();
    __shared__ float red[4];
    const int t = blockIdx.x, hb = blockIdx.y, tid = threadIdx.x, ch = hb * TV_DN + tid;
    float x[4];
    x[3] = bf2f(proj[(size_t)t * ldp + ch]);
    node_conv[(size_t)t * conv_ch + ch] = x[3];
    int a = t, cs = 2;
#pragma unroll
    for (int k = 2; k >= 0; --k) {
        if (a >= 0) a = parents[a];
        x[k] = (a >= 0) ? bf2f(proj[(size_t)a * ldp + ch]) : conv_state[(size_t)(cs--) * conv_ch + ch];
    }
    const float4 w = *reinterpret_cast<const float4*>(conv_w + (size_t)ch * 4);
    float s = w.x * x[0];
    s = fmaf(w.y, x[1], s); s = fmaf(w.z, x[2], s); s = fmaf(w.w, x[3], s);
    float y = silu_f(s);
    if (hb < 2 * D.dn_k_heads) {                              // block-uniform
        const float ss = tv_block_sum(y * y, red);
        y = y * rsqrt_ieee(ss + D.eps);
        if (hb < D.dn_k_heads) y *= 0.08838834764831845f;
    } else if (tid == 0) {
        const int h = hb - 2 * D.dn_k_heads;
        const float b = bf2f(ba[(size_t)t * ldba + h]);
        const float al = bf2f(ba[(size_t)t * ldba + D.dn_v_heads + h]) + dt_bias[h];
        const float sp = (al > 20.f) ? al : log1pf(expf(al));
        gate[((size_t)t * D.dn_v_heads + h) * 2] = sigmoid_f(b);
        gate[((size_t)t * D.dn_v_heads + h) * 2 + 1] = expf(sp * ssm_a[h]);
    }
    qkv[(size_t)t * conv_ch + ch] = y;
}

// tree gated delta rule: one CTA of 128 threads per (v head, block of 16 value rows); nodes in the given order.
// Thread (row, slice) owns 16 state elements of one value row (float4 number slice + 8 i, i = 0..3), so a row's dot
// products reduce over 8 lanes.  Every node's q, k, 16 values and gate pair are staged in shared memory up front.
// The running f32 state continues from node t-1 when that is the parent; otherwise it restarts from the parent's
// persisted f16 post-state (a thread-private copy in a shared-memory slot when tv_tree_prep planned one, else global
// memory), or from the committed f32 state for a root.  Every node's post-state is persisted as f16
// (qwen35_target_graph.cpp:540-583).  v head h uses k head h % k_heads (ggml_repeat tiling, :531-534).
__host__ __device__ constexpr size_t tv_dn_tree_smem(int n) {
    return ((size_t)n * (2 * TV_DN + 16 + 2) * 4 + (size_t)n * 3 * 4 + 15) / 16 * 16 + (size_t)TV_DN_SLOTS * 4 * 128 * 8;
}
__device__ __forceinline__ float dot4_rn(const float4& a, const float4& b) {
    return __fadd_rn(__fadd_rn(__fadd_rn(__fmul_rn(a.x, b.x), __fmul_rn(a.y, b.y)), __fmul_rn(a.z, b.z)), __fmul_rn(a.w, b.w));
}
__global__ void __launch_bounds__(128) tv_dn_tree_kernel(const float* __restrict__ qkv, int conv_ch, const float* __restrict__ gate,
                                                         const int* __restrict__ parents, const int* __restrict__ src, const int* __restrict__ save,
                                                         int n_nodes, TvDims D, const float* __restrict__ ssm_state, __half* __restrict__ node_states,
                                                         float* __restrict__ core) {
    pdl_wait();
    extern __shared__ __align__(16) unsigned char tv_smem[];
    float* sq = reinterpret_cast<float*>(tv_smem);                       // [n][128]
    float* sk = sq + (size_t)n_nodes * TV_DN;                             // [n][128]
    float* sv = sk + (size_t)n_nodes * TV_DN;                             // [n][16]
    float* sg = sv + (size_t)n_nodes * 16;                                // [n][2]
    int* sp = reinterpret_cast<int*>(sg + (size_t)n_nodes * 2);           // [n] parent, [n] source, [n] slot to keep
    int* ssrc = sp + n_nodes;
    int* ssave = ssrc + n_nodes;
    uint2* slots = reinterpret_cast<uint2*>(tv_smem + tv_dn_tree_smem(n_nodes) - (size_t)TV_DN_SLOTS * 4 * 128 * 8);   // [slot][i][thread]
    const int h = blockIdx.x, rb = blockIdx.y, tid = threadIdx.x;
    const int kh = h % D.dn_k_heads;
    const size_t head_elems = (size_t)TV_DN * TV_DN;
    for (int i = tid; i < n_nodes * (TV_DN / 4); i += 128) {
        const int t = i / (TV_DN / 4), l = i % (TV_DN / 4);
        const float* row = qkv + (size_t)t * conv_ch;
        cp_async16(sq + (size_t)t * TV_DN + l * 4, row + kh * TV_DN + l * 4);
        cp_async16(sk + (size_t)t * TV_DN + l * 4, row + (D.dn_k_heads + kh) * TV_DN + l * 4);
    }
    for (int i = tid; i < n_nodes * 4; i += 128)
        cp_async16(sv + (size_t)(i >> 2) * 16 + (i & 3) * 4, qkv + (size_t)(i >> 2) * conv_ch + 2 * D.dn_k_heads * TV_DN + h * TV_DN + rb * 16 + (i & 3) * 4);
    for (int i = tid; i < n_nodes * 2; i += 128) sg[i] = gate[((size_t)(i >> 1) * D.dn_v_heads + h) * 2 + (i & 1)];
    for (int i = tid; i < n_nodes; i += 128) { sp[i] = parents[i]; ssrc[i] = src[i]; ssave[i] = save[i]; }
    cp_async_wait_all();
    __syncthreads();
    const int rr = tid >> 3, sl = tid & 7;
    const int vrow = rb * 16 + rr;
    float4 st[4];
    for (int t = 0; t < n_nodes; ++t) {
        const int from = ssrc[t];
        if (from != -2) {
            const int p = sp[t];
            if (from >= 0) {
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const uint2 raw = slots[(from * 4 + i) * 128 + tid];
                    const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&raw.x)), b = __half22float2(*reinterpret_cast<const __half2*>(&raw.y));
                    st[i] = make_float4(a.x, a.y, b.x, b.y);
                }
            } else if (p < 0 || p >= t) {
#pragma unroll
                for (int i = 0; i < 4; ++i) st[i] = *(reinterpret_cast<const float4*>(ssm_state + (size_t)h * head_elems + (size_t)vrow * TV_DN) + sl + 8 * i);
            } else {
                uint2 raw[4];
#pragma unroll
                for (int i = 0; i < 4; ++i)
                    raw[i] = *(reinterpret_cast<const uint2*>(node_states + ((size_t)p * D.dn_v_heads + h) * head_elems + (size_t)vrow * TV_DN) + sl + 8 * i);
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&raw[i].x)), b = __half22float2(*reinterpret_cast<const __half2*>(&raw[i].y));
                    st[i] = make_float4(a.x, a.y, b.x, b.y);
                }
            }
        }
        float4 q4[4], k4[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            q4[i] = *(reinterpret_cast<const float4*>(sq + (size_t)t * TV_DN) + sl + 8 * i);
            k4[i] = *(reinterpret_cast<const float4*>(sk + (size_t)t * TV_DN) + sl + 8 * i);
        }
        const float beta = sg[2 * t], decay = sg[2 * t + 1], vv = sv[t * 16 + rr];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            st[i].x = __fmul_rn(st[i].x, decay); st[i].y = __fmul_rn(st[i].y, decay); st[i].z = __fmul_rn(st[i].z, decay); st[i].w = __fmul_rn(st[i].w, decay);
        }
        float kv = __fadd_rn(__fadd_rn(dot4_rn(st[0], k4[0]), dot4_rn(st[1], k4[1])), __fadd_rn(dot4_rn(st[2], k4[2]), dot4_rn(st[3], k4[3])));
        kv += __shfl_xor_sync(0xffffffffu, kv, 1); kv += __shfl_xor_sync(0xffffffffu, kv, 2); kv += __shfl_xor_sync(0xffffffffu, kv, 4);
        const float delta = __fmul_rn(__fsub_rn(vv, kv), beta);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            st[i].x = __fadd_rn(st[i].x, __fmul_rn(k4[i].x, delta)); st[i].y = __fadd_rn(st[i].y, __fmul_rn(k4[i].y, delta));
            st[i].z = __fadd_rn(st[i].z, __fmul_rn(k4[i].z, delta)); st[i].w = __fadd_rn(st[i].w, __fmul_rn(k4[i].w, delta));
        }
        float o = __fadd_rn(__fadd_rn(dot4_rn(st[0], q4[0]), dot4_rn(st[1], q4[1])), __fadd_rn(dot4_rn(st[2], q4[2]), dot4_rn(st[3], q4[3])));
        o += __shfl_xor_sync(0xffffffffu, o, 1); o += __shfl_xor_sync(0xffffffffu, o, 2); o += __shfl_xor_sync(0xffffffffu, o, 4);
        const int keep = ssave[t];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const __half2 h0 = __floats2half2_rn(st[i].x, st[i].y), h1 = __floats2half2_rn(st[i].z, st[i].w);
            const uint2 raw = make_uint2(*reinterpret_cast<const uint32_t*>(&h0), *reinterpret_cast<const uint32_t*>(&h1));
            *(reinterpret_cast<uint2*>(node_states + ((size_t)t * D.dn_v_heads + h) * head_elems + (size_t)vrow * TV_DN) + sl + 8 * i) = raw;
            if (keep >= 0) slots[(keep * 4 + i) * 128 + tid] = raw;
        }
        if (sl == 0) core[((size_t)t * D.dn_v_heads + h) * TV_DN + vrow] = o;
    }
}

// gated norm: y = bf16(o * rsqrt(mean o^2 + eps) * w * silu(z)).  grid (nodes, v_heads), 128 threads
__global__ void __launch_bounds__(128) tv_dn_gated_norm_kernel(const float* __restrict__ core, const bf16* __restrict__ proj, int ldp, int z_off,
                                                               const float* __restrict__ w, TvDims D, bf16* __restrict__ out) {
    pdl_trigger();      // the projection GEMM that follows loads and dequantises its first weights beside this kernel
    pdl_wait();
    __shared__ float red[4];
    const int t = blockIdx.x, h = blockIdx.y, tid = threadIdx.x;
    const float o = core[((size_t)t * D.dn_v_heads + h) * TV_DN + tid];
    const float inv = rsqrt_ieee(tv_block_sum(o * o, red) / (float)TV_DN + D.eps);
    const float z = bf2f(proj[(size_t)t * ldp + z_off + h * TV_DN + tid]);
    out[((size_t)t * D.dn_v_heads + h) * TV_DN + tid] = f2bf(o * inv * w[tid] * silu_f(z));
}

// ------------------------------------------- head and walk -------------------------------------------
// arg-max of every node's bf16 logits, lowest index among equal maxima.  grid nodes, 1024 threads
__global__ void __launch_bounds__(1024) tv_argmax_kernel(const bf16* __restrict__ logits, int vocab, int* __restrict__ out) {
    pdl_wait();
    __shared__ float sv[32];
    __shared__ int si[32];
    const bf16* row = logits + (size_t)blockIdx.x * vocab;
    float best = -INFINITY; int bi = 0x7fffffff;
    for (int i = threadIdx.x; i < vocab; i += 1024) {
        const float v = bf2f(row[i]);
        if (v > best) { best = v; bi = i; }
    }
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, best, o); const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > best || (ov == best && oi < bi)) { best = ov; bi = oi; }
    }
    if ((threadIdx.x & 31) == 0) { sv[threadIdx.x >> 5] = best; si[threadIdx.x >> 5] = bi; }
    __syncthreads();
    if (threadIdx.x < 32) {
        best = sv[threadIdx.x]; bi = si[threadIdx.x];
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, best, o); const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (ov > best || (ov == best && oi < bi)) { best = ov; bi = oi; }
        }
        if (threadIdx.x == 0) out[blockIdx.x] = bi;
    }
}

// accepted path: from the root follow the child whose token equals the arg-max of the current node
// (test_dflash.cpp:396-415).  result[0] = path length, result[1] = next token (arg-max of the last accepted node),
// path[i] = DFS index of the i-th accepted node.
__global__ void tv_accept_kernel(const int* __restrict__ tokens, const int* __restrict__ parents, const int* __restrict__ argmax, int n,
                                 int* __restrict__ path, int* __restrict__ result) {
    if (threadIdx.x != 0 || blockIdx.x != 0) return;
    int cur = 0, len = 1;
    path[0] = 0;
    for (;;) {
        const int want = argmax[cur];
        int next = -1;
        for (int c = cur + 1; c < n; ++c)
            if (parents[c] == cur && tokens[c] == want) { next = c; break; }
        if (next < 0) break;
        cur = next;
        path[len++] = cur;
    }
    result[0] = len;
    result[1] = argmax[cur];
}

// commit (test_dflash.cpp:1355-1521): recurrent state <- persisted state of the last accepted node
__global__ void tv_commit_state_kernel(const __half* __restrict__ node_states, size_t layer_stride_nodes, size_t node_elems, int n_dn,
                                       const int* __restrict__ path, const int* __restrict__ result, float* __restrict__ ssm_state) {
    const int leaf = path[result[0] - 1];
    const size_t total = (size_t)n_dn * node_elems;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        const size_t l = i / node_elems, e = i % node_elems;
        ssm_state[i] = __half2float(node_states[l * layer_stride_nodes + (size_t)leaf * node_elems + e]);
    }
}
// conv state <- the last three inputs along [old state rows 0..2, accepted nodes...]
__global__ void tv_commit_conv_kernel(const float* __restrict__ node_conv, size_t layer_stride_nodes, int conv_ch, int n_dn,
                                      const int* __restrict__ path, const int* __restrict__ result, float* __restrict__ conv_state) {
    const int len = result[0];
    const size_t total = (size_t)n_dn * conv_ch;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        const size_t l = i / conv_ch, ch = i % conv_ch;
        float* cs = conv_state + l * 3 * conv_ch;
        float old[3] = {cs[ch], cs[conv_ch + ch], cs[2 * (size_t)conv_ch + ch]};
        float nv[3];
#pragma unroll
        for (int k = 0; k < 3; ++k) {
            const int idx = len + k;                 // position in [old0, old1, old2, node path...] of new row k
            nv[k] = idx < 3 ? old[idx] : node_conv[l * layer_stride_nodes + (size_t)path[idx - 3] * conv_ch + ch];
        }
        cs[ch] = nv[0]; cs[conv_ch + ch] = nv[1]; cs[2 * (size_t)conv_ch + ch] = nv[2];
    }
}
// K/V rows of the accepted nodes move to slots past, past+1, ... (ascending, so no source is overwritten early).
// Rows are row_bytes long (512 bf16, 272 Q8_0), copied in 16-byte pieces.
__global__ void tv_commit_kv_kernel(unsigned char* __restrict__ k_cache, unsigned char* __restrict__ v_cache, size_t layer_stride, int n_fa, int kv_heads,
                                    int max_ctx, int row_bytes, int past, const int* __restrict__ path, const int* __restrict__ result) {
    const int len = result[0];
    const int per_row = row_bytes / 16;
    const size_t total = (size_t)n_fa * kv_heads * per_row * 2;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        const int c16 = (int)(i % per_row);
        const size_t rest = i / per_row;
        const int which = (int)(rest % 2);
        const size_t lh = rest / 2;                  // layer * kv_heads + head
        unsigned char* base = (which ? v_cache : k_cache) + (lh / kv_heads) * layer_stride + ((lh % kv_heads) * (size_t)max_ctx) * row_bytes + c16 * 16;
        for (int d = 0; d < len; ++d) {
            const int src = past + path[d], dst = past + d;
            if (src != dst) *reinterpret_cast<uint4*>(base + (size_t)dst * row_bytes) = *reinterpret_cast<const uint4*>(base + (size_t)src * row_bytes);
        }
    }
}

// feature capture: rows of `hidden` (node t) -> ring row (past + t) % cap, column block k.  grid nodes, 256 threads
__global__ void __launch_bounds__(256) tv_capture_kernel(const bf16* __restrict__ hidden, int H, int past, int cap, int row_elems, int col0,
                                                         bf16* __restrict__ ring) {
    pdl_wait();
    const int t = blockIdx.x;
    const uint4* src = reinterpret_cast<const uint4*>(hidden + (size_t)t * H);
    uint4* dst = reinterpret_cast<uint4*>(ring + (size_t)((past + t) % cap) * row_elems + col0);
    for (int i = threadIdx.x; i < H / 8; i += 256) dst[i] = src[i];
}
// ring rows of the accepted nodes move to positions past, past+1, ... (ascending, so no source is overwritten early;
// path[d] >= d because node numbers grow along a path)
__global__ void tv_commit_feat_kernel(bf16* __restrict__ ring, int row_elems, int cap, int past, const int* __restrict__ path, const int* __restrict__ result) {
    const int len = result[0];
    for (int d = 0; d < len; ++d) {
        const int src = (past + path[d]) % cap, dst = (past + d) % cap;
        if (src == dst) continue;
        const uint4* s = reinterpret_cast<const uint4*>(ring + (size_t)src * row_elems);
        uint4* o = reinterpret_cast<uint4*>(ring + (size_t)dst * row_elems);
        for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < row_elems / 8; i += gridDim.x * blockDim.x) o[i] = s[i];
    }
}

// ------------------------------------------------ host ------------------------------------------------
struct TvScratch {
    bf16 *hidden, *resid, *normed, *proj, *ba, *qbuf, *attn, *mlp, *logits;
    float *dn_qkv, *dn_gate, *core, *scores, *stats, *partial;
    int* depth; unsigned long long* anc; int* dn_src; int* dn_save;
    size_t bytes;
};

static size_t align_up(size_t v) { return (v + 255) & ~(size_t)255; }

static TvScratch tv_layout(const TvDims& D, int n, int max_ctx, char* base) {
    TvScratch s;
    size_t off = 0;
    auto take = [&](size_t bytes) { char* p = base ? base + off : nullptr; off += align_up(bytes); return p; };
    const int conv_ch = (2 * D.dn_k_heads + D.dn_v_heads) * TV_DN;
    const int fa_in = (2 * D.q_heads + 2 * D.kv_heads) * TV_HD, dn_in = conv_ch + D.dn_v_heads * TV_DN;
    const int proj_w = fa_in > dn_in ? fa_in : dn_in;
    const int att_w = D.q_heads * TV_HD > D.dn_v_heads * TV_DN ? D.q_heads * TV_HD : D.dn_v_heads * TV_DN;
    const int lpad = ((max_ctx + TV_CHUNK - 1) / TV_CHUNK) * TV_CHUNK, chunks = lpad / TV_CHUNK;
    s.hidden = (bf16*)take((size_t)n * D.hidden * 2); s.resid = (bf16*)take((size_t)n * D.hidden * 2); s.normed = (bf16*)take((size_t)n * D.hidden * 2);
    s.proj = (bf16*)take((size_t)n * proj_w * 2); s.ba = (bf16*)take((size_t)n * 2 * D.dn_v_heads * 2);
    s.qbuf = (bf16*)take((size_t)n * D.q_heads * TV_HD * 2); s.attn = (bf16*)take((size_t)n * att_w * 2);
    s.mlp = (bf16*)take((size_t)n * D.ffn * 2); s.logits = (bf16*)take((size_t)n * D.vocab * 2);
    s.dn_qkv = (float*)take((size_t)n * conv_ch * 4); s.dn_gate = (float*)take((size_t)n * D.dn_v_heads * 2 * 4);
    s.core = (float*)take((size_t)n * D.dn_v_heads * TV_DN * 4);
    s.scores = (float*)take((size_t)n * D.q_heads * lpad * 4); s.stats = (float*)take((size_t)n * D.q_heads * 2 * 4);
    s.partial = (float*)take((size_t)n * D.q_heads * chunks * TV_HD * 4);
    s.depth = (int*)take(64 * 4); s.anc = (unsigned long long*)take(64 * 8); s.dn_src = (int*)take(64 * 4); s.dn_save = (int*)take(64 * 4);
    s.bytes = off;
    return s;
}

static bool tv_dims_ok(const TvDims& D) {
    return D.head_dim == TV_HD && D.dn_dim == TV_DN && D.hidden % 256 == 0 && D.ffn % 256 == 0 && D.q_heads % D.kv_heads == 0 &&
           D.rot_dim % 2 == 0 && D.rot_dim <= TV_HD && D.dn_v_heads % D.dn_k_heads == 0 && D.n_layers > 0 && D.fa_period > 0 && D.vocab > 0;
}

// C[M, out_rows] = epi(X[M, in] . W[out_rows, in]^T) in one launch.  epi 2: W = [gate rows ; up rows], out = ffn.
// W is Q4_K super-blocks (dequantised in the kernel) or, when `dense`, plain bf16 [rows][in] (what a loader makes of a
// tensor stored in another quantisation type).
static int q4k_linear(const bf16* X, int lda, const void* W, bool dense, int out_rows, int in_cols, bf16* C, int ldc, const bf16* R, int ldr,
                      int M, int epi, cudaStream_t stream) {
    const int w_rows = epi == 2 ? 2 * out_rows : out_rows;
    if (dense) return gemm_bf16(X, lda, (const bf16*)W, w_rows, C, ldc, R, ldr, M, out_rows, in_cols, epi, out_rows, stream);
    return gemm_q4k(X, lda, (const uint8_t*)W, w_rows, C, ldc, R, ldr, M, out_rows, in_cols, epi, out_rows, stream);
}

// embedding rows from a dense bf16 table
__global__ void __launch_bounds__(256) tv_embed_dense_kernel(const bf16* __restrict__ embd, const int* __restrict__ tokens, int hidden, bf16* __restrict__ out) {
    pdl_wait();
    const bf16* src = embd + (size_t)tokens[blockIdx.x] * hidden;
    for (int i = threadIdx.x; i < hidden; i += 256) out[(size_t)blockIdx.x * hidden + i] = src[i];
}

}  // namespace q35

#define Q35_TRYT(expr)                       \
    do {                                     \
        const int st__ = (expr);             \
        if (st__ != QWEN35_OK) return st__;  \
    } while (0)

static q35::TvDims to_dims(const Qwen35TreeDims* d) {
    q35::TvDims D;
    D.n_layers = d->n_layers; D.hidden = d->hidden; D.ffn = d->ffn; D.vocab = d->vocab; D.q_heads = d->q_heads; D.kv_heads = d->kv_heads;
    D.head_dim = d->head_dim; D.dn_k_heads = d->dn_k_heads; D.dn_v_heads = d->dn_v_heads; D.dn_dim = d->dn_dim; D.rot_dim = d->rot_dim;
    D.fa_period = d->fa_period; D.theta = d->rope_theta; D.eps = d->rms_eps;
    return D;
}

extern "C" size_t qwen35_b200_tree_scratch_bytes(const Qwen35TreeDims* dims, int n_nodes, int max_ctx) {
    if (!dims) return 0;
    return q35::tv_layout(to_dims(dims), n_nodes, max_ctx, nullptr).bytes;
}

extern "C" int qwen35_b200_dequant_q4k(const void* blocks, size_t n_blocks, void* out_f32, void* out_bf16, qwen35_stream_t stream) {
    using namespace q35;
    if (!blocks || (!out_f32 && !out_bf16)) { set_error("dequant_q4k: null pointer"); return QWEN35_ERR_BAD_ARG; }
    if (n_blocks == 0) return QWEN35_OK;
    tv_dequant_q4k_kernel<<<(unsigned)((n_blocks + 7) / 8), 256, 0, (cudaStream_t)stream>>>((const uint8_t*)blocks, 0, n_blocks, (bf16*)out_bf16, (float*)out_f32);
    Q35_CUDA_OK(cudaGetLastError());
    g_launches.fetch_add(1);
    return QWEN35_OK;
}

extern "C" int qwen35_b200_tree_verify(const Qwen35TreeVerifyArgs* in, qwen35_stream_t stream_) {
    using namespace q35;
    cudaStream_t stream = (cudaStream_t)stream_;
    if (!in || !in->layers) { set_error("tree_verify: null args"); return QWEN35_ERR_BAD_ARG; }
    const TvDims D = to_dims(&in->dims);
    const int n = in->n_nodes;
    if (!tv_dims_ok(D)) { set_error("tree_verify: unsupported dimensions (head_dim must be 256, DeltaNet head 128, hidden and ffn multiples of 256)"); return QWEN35_ERR_BAD_ARG; }
    const int gqa = D.q_heads / D.kv_heads;
    if (n <= 0 || n > TV_MAX_NODES || n * gqa > 240) { set_error("tree_verify: %d nodes out of range (1..%d, nodes x q-per-kv <= 240)", n, TV_MAX_NODES); return QWEN35_ERR_BAD_ARG; }
    if (in->past < 0 || in->past + n > in->max_ctx) { set_error("tree_verify: past %d + %d nodes exceeds max_ctx %d", in->past, n, in->max_ctx); return QWEN35_ERR_BAD_ARG; }
    if (!in->token_embd || !in->output_norm || !in->output_w || !in->node_tokens || !in->parents || !in->k_cache || !in->v_cache || !in->ssm_state ||
        !in->conv_state || !in->node_states || !in->node_conv || !in->node_argmax || !in->scratch) {
        set_error("tree_verify: null tensor pointer");
        return QWEN35_ERR_BAD_ARG;
    }
    const TvScratch need = tv_layout(D, n, in->max_ctx, nullptr);
    if (in->scratch_bytes < need.bytes) { set_error("tree_verify: scratch of %zu bytes given, %zu needed", in->scratch_bytes, need.bytes); return QWEN35_ERR_BAD_ARG; }
    const TvScratch s = tv_layout(D, n, in->max_ctx, (char*)in->scratch);
    void* ws = get_workspace();
    if (!ws) return QWEN35_ERR_CUDA;

    const int conv_ch = (2 * D.dn_k_heads + D.dn_v_heads) * TV_DN, z_off = conv_ch;
    const int fa_in = (2 * D.q_heads + 2 * D.kv_heads) * TV_HD, dn_in = conv_ch + D.dn_v_heads * TV_DN;
    const int L = in->past + n, lpad = ((in->max_ctx + TV_CHUNK - 1) / TV_CHUNK) * TV_CHUNK;
    const int chunks = (L + TV_CHUNK - 1) / TV_CHUNK;          // chunks that hold visible keys
    const int R = n * gqa, mt_n = (R + 15) / 16;
    const size_t sc_smem = ((size_t)mt_n * 16 * TV_QSTRIDE + (size_t)TV_CHUNK * TV_QSTRIDE) * 2;
    const size_t pv_smem = ((size_t)TV_CHUNK * TV_QSTRIDE + (size_t)mt_n * 16 * TV_PSTRIDE) * 2;
    static PerDeviceOnce attr_done;
    if (attr_done.pending()) {
#define TV_ATT_SMEM(KT)                                                                                                           \
        Q35_CUDA_OK(cudaFuncSetAttribute(tv_att_scores_kernel<KT>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024)); \
        Q35_CUDA_OK(cudaFuncSetAttribute(tv_att_pv_kernel<KT>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024));
        TV_ATT_SMEM(TV_KV_BF16) TV_ATT_SMEM(TV_KV_Q8_0) TV_ATT_SMEM(TV_KV_Q4_0) TV_ATT_SMEM(TV_KV_F16)
#undef TV_ATT_SMEM
        Q35_CUDA_OK(cudaFuncSetAttribute(tv_dn_tree_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)tv_dn_tree_smem(TV_MAX_NODES)));
        attr_done.mark();
    }
    // second stream for the work that runs beside a projection; made once for the process's device and forked from /
    // joined into the caller's stream with events, so it is also legal inside a stream capture
    struct SideStream { cudaStream_t stream = nullptr; cudaEvent_t fork = nullptr, join = nullptr; };
    static SideStream side_of[64];                       // streams and events belong to a device: one set per device
    SideStream& side = side_of[PerDeviceOnce::slot()];
    if (!side.stream) {
        Q35_CUDA_OK(cudaStreamCreateWithFlags(&side.stream, cudaStreamNonBlocking));
        Q35_CUDA_OK(cudaEventCreateWithFlags(&side.fork, cudaEventDisableTiming));
        Q35_CUDA_OK(cudaEventCreateWithFlags(&side.join, cudaEventDisableTiming));
    }
    if (in->kv_type < 0 || in->kv_type > TV_KV_F16) { set_error("tree_verify: kv_type %d (0 bf16, 1 Q8_0, 2 Q4_0, 3 F16)", in->kv_type); return QWEN35_ERR_BAD_ARG; }
    const size_t kv_layer = (size_t)D.kv_heads * in->max_ctx * tv_kv_row_bytes(in->kv_type);      // bytes
    const size_t kv_raw = (size_t)tv_kv_raw_bytes(in->kv_type);
    const size_t state_layer = (size_t)D.dn_v_heads * TV_DN * TV_DN;
    const size_t nstate_layer = (size_t)in->max_nodes * state_layer, nconv_layer = (size_t)in->max_nodes * conv_ch;
    if (in->max_nodes < n) { set_error("tree_verify: max_nodes %d < n_nodes %d", in->max_nodes, n); return QWEN35_ERR_BAD_ARG; }
    if (in->target_feat && (in->feat_cap < n || in->n_capture < 1 || in->n_capture > 8)) {
        set_error("tree_verify: feature ring needs feat_cap >= n_nodes and 1..8 capture layers");
        return QWEN35_ERR_BAD_ARG;
    }

    // ~660 dependent launches per pass: programmatic dependent launch hides most of the 2-3 us between them
    PdlGuard pdl_guard;      // the Q4_K GEMM launches join in
    Q35_CUDA_OK(pdl_launch(tv_tree_prep_kernel, 1, 32, 0, stream, in->parents, n, s.depth, s.anc, s.dn_src, s.dn_save));
    if (in->dense_mask & 1u) Q35_CUDA_OK(pdl_launch(tv_embed_dense_kernel, n, 256, 0, stream, (const bf16*)in->token_embd, in->node_tokens, D.hidden, s.hidden));
    else Q35_CUDA_OK(pdl_launch(tv_embed_q4k_kernel, dim3(n, D.hidden / 256), 32, 0, stream, (const uint8_t*)in->token_embd, in->node_tokens, D.hidden, s.hidden));
    g_launches.fetch_add(2);
    const int n_layers = in->dbg_num_layers > 0 && in->dbg_num_layers < D.n_layers ? in->dbg_num_layers : D.n_layers;
    int i_fa = 0, i_dn = 0;
    for (int il = 0; il < n_layers; ++il) {
        const Qwen35TreeLayer& W = in->layers[il];
        const bool is_fa = (il % D.fa_period) == D.fa_period - 1;
        if (il > 0 && in->dbg_teacher)
            Q35_CUDA_OK(cudaMemcpyAsync(s.hidden, (const bf16*)in->dbg_teacher + (size_t)il * n * D.hidden, (size_t)n * D.hidden * 2, cudaMemcpyDeviceToDevice, stream));
        Q35_CUDA_OK(pdl_launch(tv_rmsnorm_kernel, n, 256, 0, stream, s.hidden, (const float*)W.attn_norm, s.normed, D.hidden, D.eps));
        g_launches.fetch_add(1);
        int att_w;
        if (is_fa) {
            Q35_TRYT(q4k_linear(s.normed, D.hidden, W.w_in, (W.dense_mask & 1u) != 0, fa_in, D.hidden, s.proj, fa_in, nullptr, 0, n, 0, stream));
            unsigned char* kc = (unsigned char*)in->k_cache + (size_t)i_fa * kv_layer;
            unsigned char* vc = (unsigned char*)in->v_cache + (size_t)i_fa * kv_layer;
            Q35_CUDA_OK(pdl_launch(tv_fa_prep_kernel, dim3(n, D.q_heads + 2 * D.kv_heads), 128, 0, stream, s.proj, fa_in, (const float*)W.q_norm, (const float*)W.k_norm, s.depth, D,
                                                                                       in->past, in->max_ctx, s.qbuf, kc, vc, in->kv_type));
            switch (in->kv_type) {
#define TV_SCORES(KT) case KT: Q35_CUDA_OK(pdl_launch(tv_att_scores_kernel<KT>, dim3(chunks, D.kv_heads), TV_PV_THREADS, sc_smem + kv_raw, stream, s.qbuf, kc, s.anc, D, n, in->past, in->max_ctx, lpad, s.scores)); break;
                TV_SCORES(TV_KV_BF16) TV_SCORES(TV_KV_Q8_0) TV_SCORES(TV_KV_Q4_0) TV_SCORES(TV_KV_F16)
#undef TV_SCORES
            }
            Q35_CUDA_OK(pdl_launch(tv_att_stats_kernel, (D.kv_heads * R + 7) / 8, 256, 0, stream, s.scores, D.kv_heads * R, lpad, chunks * TV_CHUNK, s.stats));
            switch (in->kv_type) {
#define TV_PV(KT) case KT: Q35_CUDA_OK(pdl_launch(tv_att_pv_kernel<KT>, dim3(chunks, D.kv_heads), TV_PV_THREADS, pv_smem + kv_raw, stream, vc, s.scores, s.stats, D, n, in->past, in->max_ctx, lpad, s.partial)); break;
                TV_PV(TV_KV_BF16) TV_PV(TV_KV_Q8_0) TV_PV(TV_KV_Q4_0) TV_PV(TV_KV_F16)
#undef TV_PV
            }
            Q35_CUDA_OK(pdl_launch(tv_att_merge_kernel, dim3(n, D.q_heads), 128, 0, stream, s.partial, s.proj, fa_in, D, n, chunks, s.attn));
            g_launches.fetch_add(5);
            att_w = D.q_heads * TV_HD;
            ++i_fa;
        } else {
            // the small beta/alpha projection (a handful of CTAs) runs beside the input projection on a second stream
            Q35_CUDA_OK(cudaEventRecord(side.fork, stream));
            Q35_CUDA_OK(cudaStreamWaitEvent(side.stream, side.fork, 0));
            Q35_TRYT(gemm_bf16(s.normed, D.hidden, (const bf16*)W.w_ba, 2 * D.dn_v_heads, s.ba, 2 * D.dn_v_heads, nullptr, 0, n, 2 * D.dn_v_heads, D.hidden, 0, 0, side.stream));
            Q35_CUDA_OK(cudaEventRecord(side.join, side.stream));
            Q35_TRYT(q4k_linear(s.normed, D.hidden, W.w_in, (W.dense_mask & 1u) != 0, dn_in, D.hidden, s.proj, dn_in, nullptr, 0, n, 0, stream));
            float* cstate = (float*)in->conv_state + (size_t)i_dn * 3 * conv_ch;
            float* nconv = (float*)in->node_conv + (size_t)i_dn * nconv_layer;
            __half* nstates = (__half*)in->node_states + (size_t)i_dn * nstate_layer;
            Q35_CUDA_OK(cudaStreamWaitEvent(stream, side.join, 0));
            Q35_CUDA_OK(pdl_launch(tv_dn_conv_norm_kernel, dim3(n, conv_ch / TV_DN), 128, 0, stream, s.proj, dn_in, in->parents, cstate, (const float*)W.conv_w, conv_ch, s.ba, 2 * D.dn_v_heads,
                                                                              (const float*)W.ssm_a, (const float*)W.dt_bias, D, s.dn_qkv, nconv, s.dn_gate));
            Q35_CUDA_OK(pdl_launch(tv_dn_tree_kernel, dim3(D.dn_v_heads, TV_DN / 16), 128, tv_dn_tree_smem(n), stream, s.dn_qkv, conv_ch, s.dn_gate, in->parents, s.dn_src, s.dn_save, n, D,
                                                                                 (const float*)in->ssm_state + (size_t)i_dn * state_layer, nstates, s.core));
            Q35_CUDA_OK(pdl_launch(tv_dn_gated_norm_kernel, dim3(n, D.dn_v_heads), 128, 0, stream, s.core, s.proj, dn_in, z_off, (const float*)W.ssm_norm, D, s.attn));
            g_launches.fetch_add(3);
            att_w = D.dn_v_heads * TV_DN;
            ++i_dn;
        }
        Q35_TRYT(q4k_linear(s.attn, att_w, W.w_out, (W.dense_mask & 2u) != 0, D.hidden, att_w, s.resid, D.hidden, s.hidden, D.hidden, n, 1, stream));
        Q35_CUDA_OK(pdl_launch(tv_rmsnorm_kernel, n, 256, 0, stream, s.resid, (const float*)W.post_norm, s.normed, D.hidden, D.eps));
        g_launches.fetch_add(1);
        Q35_TRYT(q4k_linear(s.normed, D.hidden, W.w_gate_up, (W.dense_mask & 4u) != 0, D.ffn, D.hidden, s.mlp, D.ffn, nullptr, 0, n, 2, stream));
        Q35_TRYT(q4k_linear(s.mlp, D.ffn, W.w_down, (W.dense_mask & 8u) != 0, D.hidden, D.ffn, s.hidden, D.hidden, s.resid, D.hidden, n, 1, stream));
        if (in->dbg_hidden)
            Q35_CUDA_OK(cudaMemcpyAsync((bf16*)in->dbg_hidden + (size_t)il * n * D.hidden, s.hidden, (size_t)n * D.hidden * 2, cudaMemcpyDeviceToDevice, stream));
        if (in->target_feat)
            for (int k = 0; k < in->n_capture; ++k)
                if (in->capture_layers[k] == il) {
                    Q35_CUDA_OK(pdl_launch(tv_capture_kernel, n, 256, 0, stream, s.hidden, D.hidden, in->past, in->feat_cap, in->n_capture * D.hidden, k * D.hidden, (bf16*)in->target_feat));
                    g_launches.fetch_add(1);
                }
    }
    Q35_CUDA_OK(pdl_launch(tv_rmsnorm_kernel, n, 256, 0, stream, s.hidden, (const float*)in->output_norm, s.normed, D.hidden, D.eps));
    Q35_TRYT(q4k_linear(s.normed, D.hidden, in->output_w, (in->dense_mask & 2u) != 0, D.vocab, D.hidden, s.logits, D.vocab, nullptr, 0, n, 0, stream));
    Q35_CUDA_OK(pdl_launch(tv_argmax_kernel, n, 1024, 0, stream, s.logits, D.vocab, in->node_argmax));
    g_launches.fetch_add(2);
    if (in->logits_out) Q35_CUDA_OK(cudaMemcpyAsync(in->logits_out, s.logits, (size_t)n * D.vocab * 2, cudaMemcpyDeviceToDevice, stream));
    Q35_CUDA_OK(cudaGetLastError());
    return QWEN35_OK;
}

extern "C" int qwen35_b200_tree_accept(const int* node_tokens, const int* parents, const int* node_argmax, int n_nodes, int* path, int* result,
                                       qwen35_stream_t stream) {
    using namespace q35;
    if (!node_tokens || !parents || !node_argmax || !path || !result || n_nodes <= 0 || n_nodes > 64) { set_error("tree_accept: bad arguments"); return QWEN35_ERR_BAD_ARG; }
    tv_accept_kernel<<<1, 32, 0, (cudaStream_t)stream>>>(node_tokens, parents, node_argmax, n_nodes, path, result);
    Q35_CUDA_OK(cudaGetLastError());
    g_launches.fetch_add(1);
    return QWEN35_OK;
}

extern "C" int qwen35_b200_tree_commit(const Qwen35TreeVerifyArgs* in, const int* path, const int* result, qwen35_stream_t stream_) {
    using namespace q35;
    cudaStream_t stream = (cudaStream_t)stream_;
    if (!in || !path || !result) { set_error("tree_commit: null args"); return QWEN35_ERR_BAD_ARG; }
    const TvDims D = to_dims(&in->dims);
    if (!tv_dims_ok(D)) { set_error("tree_commit: unsupported dimensions"); return QWEN35_ERR_BAD_ARG; }
    int n_fa = 0;
    for (int il = 0; il < D.n_layers; ++il) n_fa += (il % D.fa_period) == D.fa_period - 1;
    const int n_dn = D.n_layers - n_fa;
    const int conv_ch = (2 * D.dn_k_heads + D.dn_v_heads) * TV_DN;
    const size_t state_layer = (size_t)D.dn_v_heads * TV_DN * TV_DN;
    if (n_dn > 0) {
        tv_commit_state_kernel<<<148 * 4, 256, 0, stream>>>((const __half*)in->node_states, (size_t)in->max_nodes * state_layer, state_layer, n_dn, path, result, (float*)in->ssm_state);
        tv_commit_conv_kernel<<<148, 256, 0, stream>>>((const float*)in->node_conv, (size_t)in->max_nodes * conv_ch, conv_ch, n_dn, path, result, (float*)in->conv_state);
    }
    if (n_fa > 0)
        tv_commit_kv_kernel<<<(n_fa * D.kv_heads * (TV_HD / 8) * 2 + 255) / 256, 256, 0, stream>>>((unsigned char*)in->k_cache, (unsigned char*)in->v_cache,
                                                                                                 (size_t)D.kv_heads * in->max_ctx * tv_kv_row_bytes(in->kv_type), n_fa, D.kv_heads,
                                                                                                 in->max_ctx, tv_kv_row_bytes(in->kv_type), in->past, path, result);
    if (in->target_feat && in->n_capture > 0 && in->feat_cap > 0) {
        tv_commit_feat_kernel<<<8, 256, 0, stream>>>((bf16*)in->target_feat, in->n_capture * D.hidden, in->feat_cap, in->past, path, result);
        g_launches.fetch_add(1);
    }
    Q35_CUDA_OK(cudaGetLastError());
    g_launches.fetch_add(3);
    return QWEN35_OK;
}
