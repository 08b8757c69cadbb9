// DFlash draft forward (5-layer non-causal block-diffusion draft of the 27B-class target) for sm_100a.
// Follows build_draft_graph (models/qwen35_27b/src/qwen3_dflash_graph.cpp:38-166): feature fusion, then per layer
// Q from the noise rows, K/V from [target features ; noise rows], per-head RMSNorm, NEOX RoPE, non-causal attention,
// SwiGLU.  The contractions run on the tcgen05 GEMM of gemm_tcgen05.cu (cluster split-K for the 16-row ones); this file
// holds the small kernels around them and the C entry points.
//
// Data layout in the caller's scratch (T = ctx_len + q_len rows of keys):
//   X      bf16 [T][hidden]          rows 0..ctx_len-1 = target_feat (made once per call), rows ctx_len.. = norm(h) of the layer
//   kv     bf16 [T][2 * kv_dim]      one GEMM per layer over all rows of X
//   krot   bf16 [n_kv][T][128], vv bf16 [n_kv][T][128]   head-major, K normed and rotated
//   part   f32  [n_kv][chunks][rows][128] + (max, sum) per row: chunk-local attention results, merged in chunk order
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>

#include "common.cuh"
#include "norm_kernels.cuh"
#include "runtime.h"

namespace q35 {

int gemm_bf16(const bf16* A, int lda, const bf16* B, int b_rows, bf16* C, int ldc, const bf16* R, int ldr,
              int M, int N, int K, int epi, int up_row_offset, cudaStream_t stream);
int gemm_q4k(const bf16* A, int lda, const uint8_t* W, int w_rows, bf16* C, int ldc, const bf16* R, int ldr,
             int M, int N, int K, int epi, int up_row_offset, cudaStream_t stream);

constexpr int DR_HD = 128;            // head dim (rotary over all of it, NEOX pairing i <-> i + 64)
constexpr int DR_CHUNK = 128;         // keys per attention CTA
constexpr int DR_ROWS = 64;           // query rows per kv head: q_len x (q heads per kv head), padded
constexpr int DR_LD = DR_HD + 8;      // padded shared-memory row (bf16): conflict-free ldmatrix

// per-head RMSNorm (plain weight) and NEOX RoPE of one head row; 64 threads, thread i owns the pair (i, i + 64).
// theta_i = pos * base^(-2i/128) (ggml_rope_ext, GGML_ROPE_TYPE_NEOX, n_dims = head_dim, no scaling factors).
__device__ __forceinline__ void dr_norm_rope_store(const bf16* __restrict__ src, const float* __restrict__ w, float eps, float base, int pos,
                                                   bf16* __restrict__ dst, float* red) {
    const int i = threadIdx.x;
    const float x0 = bf2f(src[i]), x1 = bf2f(src[i + 64]);
    float ss = warp_sum(x0 * x0 + x1 * x1);
    if ((i & 31) == 0) red[i >> 5] = ss;
    __syncthreads();
    ss = red[0] + red[1];
    const float inv = rsqrt_ieee(ss / (float)DR_HD + eps);
    const float y0 = x0 * inv * w[i], y1 = x1 * inv * w[i + 64];
    const float theta = (float)pos * powf(base, -2.0f * (float)i / (float)DR_HD);
    const float cs = cosf(theta), sn = sinf(theta);
    dst[i] = f2bf(y0 * cs - y1 * sn);
    dst[i + 64] = f2bf(y0 * sn + y1 * cs);
}

// Q rows: grid (q_len, n_heads), 64 threads.  qraw [q_len][n_heads*128] -> qrot [q_len][n_heads][128], position ctx_len + row
__global__ void __launch_bounds__(64) dr_q_prep_kernel(const bf16* __restrict__ qraw, const float* __restrict__ q_norm, int n_heads, int ctx_len,
                                                       float eps, float base, bf16* __restrict__ qrot) {
    pdl_wait();
    __shared__ float red[2];
    const int r = blockIdx.x, h = blockIdx.y;
    const size_t off = ((size_t)r * n_heads + h) * DR_HD;
    dr_norm_rope_store(qraw + off, q_norm, eps, base, ctx_len + r, qrot + off, red);
}

// K/V rows: grid (T, n_kv), 64 threads.  kv [T][2*n_kv*128] (k heads, then v heads) -> krot, vv [n_kv][T][128]; key row j sits at position j
__global__ void __launch_bounds__(64) dr_kv_prep_kernel(const bf16* __restrict__ kv, const float* __restrict__ k_norm, int n_kv, int T, float eps,
                                                        float base, bf16* __restrict__ krot, bf16* __restrict__ vv) {
    pdl_wait();
    __shared__ float red[2];
    const int j = blockIdx.x, h = blockIdx.y;
    const bf16* row = kv + (size_t)j * 2 * n_kv * DR_HD;
    const size_t dst = ((size_t)h * T + j) * DR_HD;
    dr_norm_rope_store(row + h * DR_HD, k_norm, eps, base, j, krot + dst, red);
    const bf16* vs = row + (n_kv + h) * DR_HD;
    vv[dst + threadIdx.x] = vs[threadIdx.x];
    vv[dst + threadIdx.x + 64] = vs[threadIdx.x + 64];
}

// Non-causal attention of all query rows of one kv head against one chunk of 128 keys.  grid (chunks, n_kv), 128 threads:
// warp w owns rows 16w..16w+15 (row = query * gqa + head-in-group).  S = Q.K^T and P.V run as mma.sync m16n8k16 bf16 tiles
// (the score accumulators become the A operand of P.V without leaving registers); the chunk keeps its own maximum m,
// P = bf16(exp(s - m)), l = sum exp(s - m) in f32, and the unnormalised f32 partial; dr_attn_merge_kernel combines them.
__global__ void __launch_bounds__(128, 1) dr_attn_chunk_kernel(const bf16* __restrict__ qrot, const bf16* __restrict__ krot, const bf16* __restrict__ vv,
                                                               int n_heads, int n_kv, int q_len, int T, float scale, float* __restrict__ part,
                                                               float* __restrict__ ml) {
    pdl_wait();
    extern __shared__ __align__(16) unsigned char dr_smem[];
    bf16* Qs = reinterpret_cast<bf16*>(dr_smem);              // [DR_ROWS][DR_LD]
    bf16* Ks = Qs + DR_ROWS * DR_LD;                          // [DR_CHUNK][DR_LD]
    bf16* Vs = Ks + DR_CHUNK * DR_LD;                         // [DR_CHUNK][DR_LD]
    const int gqa = n_heads / n_kv, R = q_len * gqa;
    const int chunk = blockIdx.x, kvh = blockIdx.y, n_chunks = gridDim.x;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, c = lane & 3;
    const int j0 = chunk * DR_CHUNK;
    for (int i = tid; i < DR_ROWS * (DR_HD / 8); i += 128) {
        const int r = i / (DR_HD / 8), c8 = i % (DR_HD / 8);
        bf16* dst = Qs + r * DR_LD + c8 * 8;
        if (r < R) cp_async16(dst, qrot + ((size_t)(r / gqa) * n_heads + kvh * gqa + r % gqa) * DR_HD + c8 * 8);
        else *reinterpret_cast<uint4*>(dst) = make_uint4(0, 0, 0, 0);
    }
    for (int i = tid; i < DR_CHUNK * (DR_HD / 8); i += 128) {
        const int k = i / (DR_HD / 8), c8 = i % (DR_HD / 8);
        bf16* kd = Ks + k * DR_LD + c8 * 8;
        bf16* vd = Vs + k * DR_LD + c8 * 8;
        if (j0 + k < T) {
            cp_async16(kd, krot + ((size_t)kvh * T + j0 + k) * DR_HD + c8 * 8);
            cp_async16(vd, vv + ((size_t)kvh * T + j0 + k) * DR_HD + c8 * 8);
        } else {
            *reinterpret_cast<uint4*>(kd) = make_uint4(0, 0, 0, 0);
            *reinterpret_cast<uint4*>(vd) = make_uint4(0, 0, 0, 0);
        }
    }
    cp_async_wait_all();
    __syncthreads();

    float sacc[DR_CHUNK / 8][4];
#pragma unroll
    for (int nt = 0; nt < DR_CHUNK / 8; ++nt) { sacc[nt][0] = 0.f; sacc[nt][1] = 0.f; sacc[nt][2] = 0.f; sacc[nt][3] = 0.f; }
#pragma unroll
    for (int ks = 0; ks < DR_HD / 16; ++ks) {
        uint32_t a[4];
        ldsm_x4(a, Qs + (warp * 16 + (lane & 15)) * DR_LD + ks * 16 + (lane >> 4) * 8);
#pragma unroll
        for (int np = 0; np < DR_CHUNK / 16; ++np) {
            uint32_t b[4];
            ldsm_x4(b, Ks + (np * 16 + (lane & 7) + 8 * (lane >> 4)) * DR_LD + ks * 16 + 8 * ((lane >> 3) & 1));
            mma_16816(sacc[2 * np], a, b[0], b[1]);
            mma_16816(sacc[2 * np + 1], a, b[2], b[3]);
        }
    }
    // scale, mask the keys past the end, chunk maximum and sum of this thread's two rows (g and g + 8)
    float m0 = -INFINITY, m1 = -INFINITY;
#pragma unroll
    for (int nt = 0; nt < DR_CHUNK / 8; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int j = j0 + nt * 8 + 2 * c + (e & 1);
            const float s = (j < T) ? sacc[nt][e] * scale : -INFINITY;
            sacc[nt][e] = s;
            if (e < 2) m0 = fmaxf(m0, s); else m1 = fmaxf(m1, s);
        }
    m0 = fmaxf(m0, __shfl_xor_sync(0xffffffffu, m0, 1)); m0 = fmaxf(m0, __shfl_xor_sync(0xffffffffu, m0, 2));
    m1 = fmaxf(m1, __shfl_xor_sync(0xffffffffu, m1, 1)); m1 = fmaxf(m1, __shfl_xor_sync(0xffffffffu, m1, 2));
    float l0 = 0.f, l1 = 0.f;
    float o[DR_HD / 8][4];
#pragma unroll
    for (int nt = 0; nt < DR_HD / 8; ++nt) { o[nt][0] = 0.f; o[nt][1] = 0.f; o[nt][2] = 0.f; o[nt][3] = 0.f; }
#pragma unroll
    for (int ks = 0; ks < DR_CHUNK / 16; ++ks) {
        uint32_t a[4];
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
            const float* sv = sacc[2 * ks + hf];
            const float p00 = (sv[0] == -INFINITY) ? 0.f : expf(sv[0] - m0), p01 = (sv[1] == -INFINITY) ? 0.f : expf(sv[1] - m0);
            const float p10 = (sv[2] == -INFINITY) ? 0.f : expf(sv[2] - m1), p11 = (sv[3] == -INFINITY) ? 0.f : expf(sv[3] - m1);
            l0 += p00 + p01; l1 += p10 + p11;
            const __nv_bfloat162 x0 = __floats2bfloat162_rn(p00, p01), x1 = __floats2bfloat162_rn(p10, p11);
            a[2 * hf] = *reinterpret_cast<const uint32_t*>(&x0);
            a[2 * hf + 1] = *reinterpret_cast<const uint32_t*>(&x1);
        }
#pragma unroll
        for (int np = 0; np < DR_HD / 16; ++np) {
            uint32_t b[4];
            ldsm_x4_trans(b, Vs + (ks * 16 + (lane & 7) + 8 * ((lane >> 3) & 1)) * DR_LD + np * 16 + 8 * (lane >> 4));
            mma_16816(o[2 * np], a, b[0], b[1]);
            mma_16816(o[2 * np + 1], a, b[2], b[3]);
        }
    }
    l0 += __shfl_xor_sync(0xffffffffu, l0, 1); l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 1); l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
        const int r = warp * 16 + g + 8 * hf;
        if (r >= R) continue;
        const size_t slot = ((size_t)kvh * n_chunks + chunk) * R + r;
        float* dst = part + slot * DR_HD;
#pragma unroll
        for (int nt = 0; nt < DR_HD / 8; ++nt)
            *reinterpret_cast<float2*>(dst + nt * 8 + 2 * c) = make_float2(o[nt][2 * hf], o[nt][2 * hf + 1]);
        if (c == 0) { ml[2 * slot] = hf ? m1 : m0; ml[2 * slot + 1] = hf ? l1 : l0; }
    }
}

// out[q][head][d] = bf16( sum_c e^(m_c - M) part_c[d] / sum_c e^(m_c - M) l_c ), chunks in ascending order.  grid (q_len, n_heads), 128 threads
__global__ void __launch_bounds__(128) dr_attn_merge_kernel(const float* __restrict__ part, const float* __restrict__ ml, int n_heads, int n_kv, int q_len,
                                                            int n_chunks, bf16* __restrict__ out) {
    pdl_wait();
    const int qi = blockIdx.x, head = blockIdx.y, d = threadIdx.x;
    const int gqa = n_heads / n_kv, kvh = head / gqa, R = q_len * gqa, r = qi * gqa + head % gqa;
    float M = -INFINITY;
    for (int ch = 0; ch < n_chunks; ++ch) M = fmaxf(M, ml[2 * (((size_t)kvh * n_chunks + ch) * R + r)]);
    float acc = 0.f, den = 0.f;
    for (int ch = 0; ch < n_chunks; ++ch) {
        const size_t slot = ((size_t)kvh * n_chunks + ch) * R + r;
        const float wgt = expf(ml[2 * slot] - M);
        acc = fmaf(wgt, part[slot * DR_HD + d], acc);
        den = fmaf(wgt, ml[2 * slot + 1], den);
    }
    out[((size_t)qi * n_heads + head) * DR_HD + d] = f2bf(acc / den);
}

// ------------------------------------------------- host side -------------------------------------------------
struct DrScratch {
    bf16 *feat_raw, *X, *h0, *h1, *qraw, *kv, *qrot, *krot, *vv, *attn, *hf, *mlp;
    float *part, *ml;
    size_t bytes;
};

static DrScratch dr_layout(const Qwen35DraftDims& D, int ctx, char* base) {
    DrScratch s;
    size_t off = 0;
    auto take = [&](size_t bytes) { char* p = base ? base + off : nullptr; off += (bytes + 255) / 256 * 256; return p; };
    const int q = D.q_len, H = D.hidden, T = ctx + q, qd = D.n_heads * DR_HD, kvd = D.n_kv_heads * DR_HD;
    const int chunks = (T + DR_CHUNK - 1) / DR_CHUNK, R = q * (D.n_heads / D.n_kv_heads);
    s.feat_raw = (bf16*)take((size_t)ctx * H * 2); s.X = (bf16*)take((size_t)T * H * 2);
    s.h0 = (bf16*)take((size_t)q * H * 2); s.h1 = (bf16*)take((size_t)q * H * 2);
    s.qraw = (bf16*)take((size_t)q * qd * 2); s.kv = (bf16*)take((size_t)T * 2 * kvd * 2); s.qrot = (bf16*)take((size_t)q * qd * 2);
    s.krot = (bf16*)take((size_t)T * kvd * 2); s.vv = (bf16*)take((size_t)T * kvd * 2);
    s.attn = (bf16*)take((size_t)q * qd * 2); s.hf = (bf16*)take((size_t)q * H * 2); s.mlp = (bf16*)take((size_t)q * D.inter * 2);
    s.part = (float*)take((size_t)D.n_kv_heads * chunks * R * DR_HD * 4); s.ml = (float*)take((size_t)D.n_kv_heads * chunks * R * 2 * 4);
    s.bytes = off;
    return s;
}

static bool dr_dims_ok(const Qwen35DraftDims& D) {
    return D.head_dim == DR_HD && D.n_layers > 0 && D.n_heads > 0 && D.n_kv_heads > 0 && D.n_heads % D.n_kv_heads == 0 && D.q_len > 0 &&
           D.q_len * (D.n_heads / D.n_kv_heads) <= DR_ROWS && D.hidden % 256 == 0 && D.inter % 256 == 0 && D.n_target_layers > 0;
}

}  // namespace q35

#define Q35_TRYD(expr)                         \
    do {                                       \
        const int rc__ = (expr);               \
        if (rc__ != QWEN35_OK) return rc__;    \
    } while (0)

extern "C" size_t qwen35_b200_draft_scratch_bytes(const Qwen35DraftDims* dims, int max_ctx_len) {
    using namespace q35;
    if (!dims || !dr_dims_ok(*dims) || max_ctx_len < 0) return 0;
    return dr_layout(*dims, max_ctx_len, nullptr).bytes;
}

extern "C" int qwen35_b200_draft_forward(const Qwen35DraftArgs* in) {
    using namespace q35;
    if (!in || !in->layers || !in->fc || !in->hidden_norm || !in->out_norm || !in->noise_embed || !in->hidden_out || !in->scratch) {
        set_error("draft_forward: null argument");
        return QWEN35_ERR_BAD_ARG;
    }
    const Qwen35DraftDims& D = in->dims;
    if (!dr_dims_ok(D)) { set_error("draft_forward: unsupported dims (head_dim 128, q_len x gqa <= 64, hidden and inter multiples of 256)"); return QWEN35_ERR_BAD_ARG; }
    const int ctx = in->ctx_len;
    if (ctx < 0 || (ctx > 0 && !in->target_hidden_cat)) { set_error("draft_forward: bad ctx_len / target_hidden_cat"); return QWEN35_ERR_BAD_ARG; }
    if (in->lm_head && (!in->logits_out || in->vocab <= 0)) { set_error("draft_forward: lm_head needs logits_out and vocab"); return QWEN35_ERR_BAD_ARG; }
    const DrScratch s = dr_layout(D, ctx, (char*)in->scratch);
    if (in->scratch_bytes < s.bytes) { set_error("draft_forward: scratch %zu < %zu bytes", in->scratch_bytes, s.bytes); return QWEN35_ERR_BAD_ARG; }
    cudaStream_t stream = (cudaStream_t)in->stream;
    const int q = D.q_len, H = D.hidden, T = ctx + q, qd = D.n_heads * DR_HD, kvd = D.n_kv_heads * DR_HD, fc_in = D.n_target_layers * H;
    const int chunks = (T + DR_CHUNK - 1) / DR_CHUNK;
    const size_t att_smem = (size_t)(DR_ROWS + 2 * DR_CHUNK) * DR_LD * 2;
    static PerDeviceOnce attr_done;
    if (attr_done.pending()) {
        Q35_CUDA_OK(cudaFuncSetAttribute(dr_attn_chunk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)att_smem));
        attr_done.mark();
    }
    PdlGuard pdl_guard;      // every kernel of the forward starts with pdl_wait(): launches overlap their predecessor's drain
    // 1. feature fusion, once per call: target_feat = rms_norm(fc . target_hidden_cat) * hidden_norm -> rows 0..ctx-1 of X
    if (ctx > 0) {
        Q35_TRYD(gemm_bf16((const bf16*)in->target_hidden_cat, fc_in, (const bf16*)in->fc, H, s.feat_raw, H, nullptr, 0, ctx, H, fc_in, 0, 0, stream));
        Q35_CUDA_OK(pdl_launch(tv_rmsnorm_kernel, ctx, 256, 0, stream, s.feat_raw, (const float*)in->hidden_norm, s.X, H, D.eps));
        g_launches.fetch_add(1);
    }
    Q35_CUDA_OK(cudaMemcpyAsync(s.h0, in->noise_embed, (size_t)q * H * 2, cudaMemcpyDeviceToDevice, stream));
    bf16 *h = s.h0, *h_next = s.h1;
    bf16* hn = s.X + (size_t)ctx * H;                          // the noise rows follow the feature rows: one K/V GEMM covers both
    const float scale = 1.0f / sqrtf((float)DR_HD);
    for (int il = 0; il < D.n_layers; ++il) {
        const Qwen35DraftLayer& L = in->layers[il];
        if (!L.attn_norm || !L.wq || !L.wkv || !L.q_norm || !L.k_norm || !L.wo || !L.ffn_norm || !L.w_gate_up || !L.w_down) {
            set_error("draft_forward: layer %d has a null weight", il);
            return QWEN35_ERR_BAD_ARG;
        }
        Q35_CUDA_OK(pdl_launch(tv_rmsnorm_kernel, q, 256, 0, stream, h, (const float*)L.attn_norm, hn, H, D.eps));
        Q35_TRYD(gemm_bf16(hn, H, (const bf16*)L.wq, qd, s.qraw, qd, nullptr, 0, q, qd, H, 0, 0, stream));
        Q35_TRYD(gemm_bf16(s.X, H, (const bf16*)L.wkv, 2 * kvd, s.kv, 2 * kvd, nullptr, 0, T, 2 * kvd, H, 0, 0, stream));
        Q35_CUDA_OK(pdl_launch(dr_q_prep_kernel, dim3(q, D.n_heads), 64, 0, stream, s.qraw, (const float*)L.q_norm, D.n_heads, ctx, D.eps, D.rope_theta, s.qrot));
        Q35_CUDA_OK(pdl_launch(dr_kv_prep_kernel, dim3(T, D.n_kv_heads), 64, 0, stream, s.kv, (const float*)L.k_norm, D.n_kv_heads, T, D.eps, D.rope_theta, s.krot, s.vv));
        Q35_CUDA_OK(pdl_launch(dr_attn_chunk_kernel, dim3(chunks, D.n_kv_heads), 128, att_smem, stream, s.qrot, s.krot, s.vv, D.n_heads, D.n_kv_heads, q, T, scale, s.part, s.ml));
        Q35_CUDA_OK(pdl_launch(dr_attn_merge_kernel, dim3(q, D.n_heads), 128, 0, stream, s.part, s.ml, D.n_heads, D.n_kv_heads, q, chunks, s.attn));
        Q35_TRYD(gemm_bf16(s.attn, qd, (const bf16*)L.wo, H, h_next, H, h, H, q, H, qd, 1, 0, stream));
        { bf16* t = h; h = h_next; h_next = t; }
        Q35_CUDA_OK(pdl_launch(tv_rmsnorm_kernel, q, 256, 0, stream, h, (const float*)L.ffn_norm, s.hf, H, D.eps));
        Q35_TRYD(gemm_bf16(s.hf, H, (const bf16*)L.w_gate_up, 2 * D.inter, s.mlp, D.inter, nullptr, 0, q, D.inter, H, 2, D.inter, stream));
        Q35_TRYD(gemm_bf16(s.mlp, D.inter, (const bf16*)L.w_down, H, h_next, H, h, H, q, H, D.inter, 1, 0, stream));
        { bf16* t = h; h = h_next; h_next = t; }
        g_launches.fetch_add(6);
    }
    Q35_CUDA_OK(pdl_launch(tv_rmsnorm_kernel, q, 256, 0, stream, h, (const float*)in->out_norm, (bf16*)in->hidden_out, H, D.eps));
    g_launches.fetch_add(1);
    if (in->lm_head) {
        if (in->lm_head_q4k)
            Q35_TRYD(gemm_q4k((const bf16*)in->hidden_out, H, (const uint8_t*)in->lm_head, in->vocab, (bf16*)in->logits_out, in->vocab, nullptr, 0, q, in->vocab, H, 0, 0, stream));
        else
            Q35_TRYD(gemm_bf16((const bf16*)in->hidden_out, H, (const bf16*)in->lm_head, in->vocab, (bf16*)in->logits_out, in->vocab, nullptr, 0, q, in->vocab, H, 0, 0, stream));
    }
    Q35_CUDA_OK(cudaGetLastError());
    return QWEN35_OK;
}
