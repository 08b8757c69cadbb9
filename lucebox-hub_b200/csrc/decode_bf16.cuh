// Device-side building blocks of the BF16 decode megakernel: per-CTA GEMV over a contiguous
// row range, RMSNorm into shared memory, and the layer stages.  Included by decode_bf16.cu.
//
// Numerics follow a bf16 HuggingFace model (the reference's declared ground truth,
// models/qwen35_0p8b/final_bench.py:241-304): every projection accumulates in f32 and is
// rounded to bf16 once, norms run in f32 and round once, the DeltaNet recurrence is f32.
#pragma once

#include "common.cuh"

namespace q35 {

constexpr int MAX_CTX = 32768;          // longest context the decode scratch is sized for
constexpr int ATT_MAX_CHUNKS = 8;       // split-KV factor of decode attention

// Library-owned scratch, one per device.  Everything a stage hands to the next stage is bf16,
// exactly as between two modules of the bf16 model.
struct Workspace {
    unsigned bar_counter;
    unsigned bar_gen;
    int err;
    int pad0[61];
    alignas(256) bf16 xa[8448];                     // stage A: DN [qkv 6144 | z 2048 | b 16 | a 16], FA [q|gate 4096 | k 512 | v 512]
    alignas(256) bf16 o[DN_V_SIZE];                 // DeltaNet core output before the gated norm
    alignas(256) bf16 h1[HIDDEN];                   // hidden after the token-mixer residual
    alignas(256) bf16 m[INTER];                     // silu(gate) * up
    alignas(256) bf16 h2[HIDDEN];                   // hidden after the MLP residual = layer output
    alignas(256) float att_part[ATT_MAX_CHUNKS][FA_Q_HEADS][FA_HEAD_DIM];
    alignas(256) float lm_val[1024];
    alignas(256) int lm_idx[1024];
    alignas(256) float scores[FA_Q_HEADS][MAX_CTX];
};

struct DecodeArgs {
    const LayerRec* layers;
    const bf16* embed;
    const bf16* final_norm;
    const bf16* lm_head;
    bf16* k_cache;
    bf16* v_cache;
    float* dn_states;
    float* conv_bufs;
    Workspace* ws;
    const int* token_in;      // device pointer to the first input token, or null -> token_imm
    int token_imm;
    const int* forced_ids;    // optional [n_steps]: input token of every step (prefill / teacher forcing)
    int* out_token;           // [1] arg-max of the last step
    int* out_tokens;          // optional [n_steps] arg-max of every step that ran the LM head
    float* logits_out;        // optional [VOCAB] (last step) bf16-rounded logits widened to f32
    bf16* hidden_out;         // optional [HIDDEN]: last layer's output of the last step
    bf16* dbg_hidden;         // optional [NUM_LAYERS][HIDDEN]: every layer's output of the last step
    const bf16* dbg_teacher;  // optional [NUM_LAYERS][HIDDEN]: input of layer l>0 is row l instead of the previous layer's output
    int position;             // tokens already cached
    int max_seq_len;
    int n_steps;
    int lm_last_only;         // 1: LM head only after the last step (prefill)
    int dbg_num_layers;       // 0 = all; otherwise stop after this many layers (debug reads of the workspace)
};

// ---- GEMV over rows [u_begin, u_end) owned by this CTA ------------------------------------------
// K: row length, WPR: warps that split one row along K, RIF: units in flight per warp,
// NMAT: matrices read per unit (2 for the gate/up pair).  rowptr(u, m) -> start of the row;
// epi(u, sums[NMAT]) is called by one thread per unit with the f32 dot products.
template <int K, int WPR, int RIF, int NMAT, typename RowFn, typename Epi>
__device__ __forceinline__ void cta_gemv(int u_begin, int u_end, const bf16* xs, float* s_part,
                                         RowFn rowptr, Epi epi) {
    constexpr int GROUPS = NWARPS / WPR;
    constexpr int KS = K / WPR;
    static_assert(KS % 256 == 0, "k-slice must be a whole number of warp-wide 16-byte chunks");
    constexpr int CPL = KS / 256;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int ks = warp % WPR, grp = warp / WPR;

    // The activation slice of this warp stays in registers for the whole stage: widened to f32
    // when it is short, packed bf16 pairs (unpacked inside the FMA loop) when it is long.
    constexpr bool PACKED = (CPL > 4);
    float x[PACKED ? 1 : CPL * 8];
    uint4 xp[PACKED ? CPL : 1];
#pragma unroll
    for (int j = 0; j < CPL; ++j) {
        const uint4 v = *reinterpret_cast<const uint4*>(xs + ks * KS + (j * 32 + lane) * 8);
        if (PACKED) {
            xp[j] = v;
        } else {
            x[j * 8 + 0] = bf_lo(v.x); x[j * 8 + 1] = bf_hi(v.x);
            x[j * 8 + 2] = bf_lo(v.y); x[j * 8 + 3] = bf_hi(v.y);
            x[j * 8 + 4] = bf_lo(v.z); x[j * 8 + 5] = bf_hi(v.z);
            x[j * 8 + 6] = bf_lo(v.w); x[j * 8 + 7] = bf_hi(v.w);
        }
    }

    for (int u = u_begin + grp; u < u_end; u += GROUPS * RIF) {
        uint4 w[RIF][NMAT][CPL];
#pragma unroll
        for (int r = 0; r < RIF; ++r) {
            const int uu = u + r * GROUPS;
            if (uu < u_end) {
#pragma unroll
                for (int m = 0; m < NMAT; ++m) {
                    const uint4* p = rowptr(uu, m) + ks * (KS / 8) + lane;
#pragma unroll
                    for (int j = 0; j < CPL; ++j) w[r][m][j] = ld_stream(p + j * 32);
                }
            }
        }
#pragma unroll
        for (int r = 0; r < RIF; ++r) {
            const int uu = u + r * GROUPS;
            if (uu < u_end) {
                float acc[NMAT];
#pragma unroll
                for (int m = 0; m < NMAT; ++m) {
                    float a = 0.f;
#pragma unroll
                    for (int j = 0; j < CPL; ++j) {
                        const uint4 q = w[r][m][j];
                        if (PACKED) {
                            const uint4 y = xp[j];
                            a = fmaf(bf_lo(q.x), bf_lo(y.x), a); a = fmaf(bf_hi(q.x), bf_hi(y.x), a);
                            a = fmaf(bf_lo(q.y), bf_lo(y.y), a); a = fmaf(bf_hi(q.y), bf_hi(y.y), a);
                            a = fmaf(bf_lo(q.z), bf_lo(y.z), a); a = fmaf(bf_hi(q.z), bf_hi(y.z), a);
                            a = fmaf(bf_lo(q.w), bf_lo(y.w), a); a = fmaf(bf_hi(q.w), bf_hi(y.w), a);
                        } else {
                            a = fmaf(bf_lo(q.x), x[j * 8 + 0], a); a = fmaf(bf_hi(q.x), x[j * 8 + 1], a);
                            a = fmaf(bf_lo(q.y), x[j * 8 + 2], a); a = fmaf(bf_hi(q.y), x[j * 8 + 3], a);
                            a = fmaf(bf_lo(q.z), x[j * 8 + 4], a); a = fmaf(bf_hi(q.z), x[j * 8 + 5], a);
                            a = fmaf(bf_lo(q.w), x[j * 8 + 6], a); a = fmaf(bf_hi(q.w), x[j * 8 + 7], a);
                        }
                    }
                    acc[m] = warp_sum(a);
                }
                if (WPR == 1) {
                    if (lane == 0) epi(uu, acc);
                } else if (lane == 0) {
#pragma unroll
                    for (int m = 0; m < NMAT; ++m) s_part[((uu - u_begin) * NMAT + m) * WPR + ks] = acc[m];
                }
            }
        }
    }
    if (WPR > 1) {
        __syncthreads();
        for (int t = threadIdx.x; t < u_end - u_begin; t += NTHREADS) {
            float acc[NMAT];
#pragma unroll
            for (int m = 0; m < NMAT; ++m) {
                float a = 0.f;
#pragma unroll
                for (int s = 0; s < WPR; ++s) a += s_part[(t * NMAT + m) * WPR + s];
                acc[m] = a;
            }
            epi(u_begin + t, acc);
        }
    }
}

// RMSNorm(1+w) of a [HIDDEN] bf16 vector into shared memory (bf16), f32 math, one rounding.
__device__ __forceinline__ void rmsnorm_to_smem(const bf16* h, const bf16* w, bf16* xs, float* s_red) {
    const int t = threadIdx.x;
    const uint32_t pr = ld_cg(reinterpret_cast<const uint32_t*>(h) + t);
    const float x0 = bf_lo(pr), x1 = bf_hi(pr);
    const float tot = block_sum(x0 * x0 + x1 * x1, s_red);
    const float r = rsqrt_ieee(tot * (1.0f / HIDDEN) + RMS_EPS);
    const uint32_t wr = __ldg(reinterpret_cast<const uint32_t*>(w) + t);
    const float y0 = (x0 * r) * (1.0f + bf_lo(wr));
    const float y1 = (x1 * r) * (1.0f + bf_hi(wr));
    reinterpret_cast<__nv_bfloat162*>(xs)[t] = __halves2bfloat162(f2bf(y0), f2bf(y1));
}

// Depthwise causal conv (kernel 4) + SiLU for one channel, given the three previous inputs in
// st.y, st.z, st.w and the new input x.  Product-sum in f32, rounded to bf16, SiLU, rounded.
__device__ __forceinline__ float conv_silu(const bf16* conv_w, int ch, float4 st, float x) {
    const uint2 wr = __ldg(reinterpret_cast<const uint2*>(conv_w) + ch);
    float c = bf_lo(wr.x) * st.y;
    c = fmaf(bf_hi(wr.x), st.z, c);
    c = fmaf(bf_lo(wr.y), st.w, c);
    c = fmaf(bf_hi(wr.y), x, c);
    c = rbf(c);
    return rbf(silu_f(c));
}

}  // namespace q35
