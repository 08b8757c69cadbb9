// Host orchestration of the BF16 prefill: per layer RMSNorm -> fused projection GEMM (tcgen05) ->
// DeltaNet (prep, chunk-local solve, scan over chunks, gated norm) or attention (q/k norm + RoPE +
// KV fill, causal attention) -> output GEMM + residual -> RMSNorm -> gate/up GEMM with fused
// SiLU*up -> down GEMM + residual; then the last token's final norm and LM-head arg-max.
//
// Replaces launch_prefill_bf16 / launch_prefill_bf16_impl of the reference (prefill.cu:1158-1497,
// declared torch_bindings.cpp:323-335).  Nothing here synchronises or copies to the host, so the
// call can be captured in a CUDA graph once the library scratch has reached its size (first call).
#include "prefill_kernels.cuh"

#include <cstdlib>

#include <cmath>
#include <mutex>

#include "runtime.h"

namespace q35 {

int gemm_bf16(const bf16* A, int lda, const bf16* B, int b_rows, bf16* C, int ldc, const bf16* R, int ldr,
              int M, int N, int K, int epi, int up_row_offset, cudaStream_t stream);
int quantize_act_nvfp4(const bf16* x, int tokens, int K, void* packed_out, void* scales_out, cudaStream_t stream);
size_t attention_tcgen05_scratch_bytes(int S);
int attention_prefill_tcgen05(const bf16* q, const bf16* k_cache, const bf16* v_cache, const bf16* proj, int ldp, bf16* out, bf16* vt_scratch, int S,
                              int max_seq, cudaStream_t stream);
int gemm_nvfp4(const void* a_packed, const void* a_scales, int tokens, const void* w_packed, const void* w_scales, int n_rows, int n_out, int K,
               float alpha, void* C, int ldc, int out_f32, const bf16* R, int ldr, cudaStream_t stream);

// grow-only per-device scratch for the chunk-local results
static void* g_scratch[64] = {};
static size_t g_scratch_bytes[64] = {};
static std::mutex g_scratch_mu;

static void* get_scratch(size_t bytes) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return nullptr;
    dev &= 63;
    std::lock_guard<std::mutex> lk(g_scratch_mu);
    if (g_scratch_bytes[dev] < bytes) {
        if (g_scratch[dev]) { cudaDeviceSynchronize(); cudaFree(g_scratch[dev]); g_scratch[dev] = nullptr; g_scratch_bytes[dev] = 0; }
        if (cudaMalloc(&g_scratch[dev], bytes) != cudaSuccess) { set_error("prefill scratch allocation of %zu bytes failed", bytes); return nullptr; }
        g_scratch_bytes[dev] = bytes;
    }
    return g_scratch[dev];
}

struct PrefillArgs {
    const int* token_ids; int S; int* out_token;
    const bf16* embed; const LayerRec* layers_host; const PrefillFused* fused_host;
    const bf16* final_norm; const bf16* lm_head;
    bf16* k_cache; bf16* v_cache; float* dn_states; float* conv_bufs;
    bf16 *hidden, *residual, *normalized, *proj_buf, *proj_buf2, *attn_buf, *mlp_buf, *dn_out_buf;
    float *beta_buf, *alpha_buf;
    bf16 *final_normed, *hidden_out;
    float* lm_bmv; int* lm_bmi;
    float* logits_out;
    const void* lm_packed;     // optional NVFP4 LM head (tensor-core layout) for the last token
    const void* lm_scales;
    const bf16* dbg_teacher;   // optional [layers][S][HIDDEN]: input of layer l > 0
    bf16* dbg_hidden;          // optional [layers][HIDDEN]: last position's output of every layer
    int max_seq_len;
    int n_layers;
};

#define Q35_TRY(expr)                        \
    do {                                     \
        const int st__ = (expr);             \
        if (st__ != QWEN35_OK) return st__;  \
    } while (0)

static int prefill_impl(const PrefillArgs& a, cudaStream_t stream) {
    const int S = a.S;
    static PerDeviceOnce attr_done;
    if (attr_done.pending()) {
        Q35_CUDA_OK(cudaFuncSetAttribute(pf_dn_chunk_local_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, CHUNK_LOCAL_SMEM));
        Q35_CUDA_OK(cudaFuncSetAttribute(pf_dn_chunk_scan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, CHUNK_SCAN_SMEM));
        attr_done.mark();
    }
    const int nchunks = (S + DN_CHUNK - 1) / DN_CHUNK;
    int* err_word = (int*)get_workspace();            // the device status word the bounded waits report to
    if (!err_word) return QWEN35_ERR_CUDA;
    // library scratch: the chunk-local results, then the NVFP4 operand of the activations (packed rows padded to 128 + scale
    // atoms) and one row of bf16 logits for the tensor-core FP4 head
    const size_t chunk_bytes = ((size_t)DN_HEADS * nchunks * sizeof(ChunkScratch) + 255) & ~(size_t)255;
    const size_t tpad = ((size_t)S + 127) / 128 * 128;
    const int s_pad = (int)tpad;               // rows of the packed NVFP4 activation operand
    const size_t act_packed_bytes = tpad * (HIDDEN / 2), act_scale_bytes = tpad / 128 * (HIDDEN / 64) * 512;
    const size_t head_bytes = (chunk_bytes + act_packed_bytes + act_scale_bytes + (size_t)VOCAB * 2 + 256 + 1023) & ~(size_t)1023;
    char* scratch_base = (char*)get_scratch(head_bytes + attention_tcgen05_scratch_bytes(S) + 1024);
    if (!scratch_base) return QWEN35_ERR_CUDA;
    ChunkScratch* scratch = (ChunkScratch*)scratch_base;
    uint8_t* act_packed = (uint8_t*)scratch_base + chunk_bytes;
    uint8_t* act_scales = act_packed + act_packed_bytes;
    bf16* lm_logits = (bf16*)(act_scales + ((act_scale_bytes + 255) & ~(size_t)255));
    bf16* vt_scratch = (bf16*)(((uintptr_t)scratch_base + head_bytes + 1023) & ~(uintptr_t)1023);     // V^T of the attention layer in flight
    RopeTable rt;
    for (int i = 0; i < FA_ROT / 2; ++i) rt.f[i] = 1.0f / (float)std::pow(1.0e7, (double)((float)(2 * i) / (float)FA_ROT));

    int i_dn = 0, i_fa = 0;
    // ~250 dependent launches per prompt: programmatic dependent launch (every kernel of the pass starts with pdl_wait())
    PdlGuard pdl_guard;
    for (int layer = 0; layer < a.n_layers; ++layer) {
        const LayerRec& L = a.layers_host[layer];
        // Without fused tables (launch_prefill_bf16_mega) every matrix of the layer record is its own GEMM, written into the
        // same column blocks of proj_buf the fused projection fills, and SiLU * up is a kernel of its own.
        const PrefillFused* F = a.fused_host ? &a.fused_host[layer] : nullptr;
        // NVFP4 copies of the two fused matrices present: their GEMMs run block-scaled on FP4 operands (activations quantised
        // per 16-element block on the way), as the reference does when its table carries them (prefill.cu:1210-1218)
        const bool fp4 = F && F->proj_packed && F->proj_scales && F->gate_up_packed && F->gate_up_scales;
        // input norm (layer 0 gathers the embedding rows into `hidden` on the way); with a teacher, layer l > 0 takes its
        // input (and the residual of its mixer) from the teacher's row block instead of the previous layer's output
        const bf16* layer_in = (a.dbg_teacher && layer > 0) ? a.dbg_teacher + (size_t)layer * S * HIDDEN : a.hidden;
        // (NVFP4: the kernel packs the normalised rows as the activation operand on the way out, and the bf16 copy is not written)
        Q35_CUDA_OK(pdl_launch(pf_rmsnorm_kernel<false>, fp4 ? s_pad : S, 128, 0, stream, layer == 0 ? a.token_ids : nullptr, a.embed, layer_in, (const bf16*)L.p[0],
                                                 layer == 0 ? a.hidden : nullptr, fp4 ? (bf16*)nullptr : a.normalized, S,
                                                 fp4 ? (uint8_t*)act_packed : (uint8_t*)nullptr, fp4 ? (uint8_t*)act_scales : (uint8_t*)nullptr));
        g_launches.fetch_add(1);
        const bf16 *w_out, *w_post, *w_down;
        if (L.type == 0) {
            const int ldp = DN_PROJ_ROWS;
            if (fp4) {
                Q35_TRY(gemm_nvfp4(act_packed, act_scales, S, F->proj_packed, F->proj_scales, (DN_PROJ_ROWS + 127) / 128 * 128, DN_PROJ_ROWS, HIDDEN, 1.0f,
                                   a.proj_buf, ldp, 0, nullptr, 0, stream));
            } else if (F) {
                Q35_TRY(gemm_bf16(a.normalized, HIDDEN, (const bf16*)F->proj_weight, DN_PROJ_ROWS, a.proj_buf, ldp, nullptr, 0, S, DN_PROJ_ROWS, HIDDEN, 0, 0, stream));
            } else {
                const int slot[4] = {DN_QKV, DN_Z, DN_B, DN_A}, rows[4] = {DN_CONV_CH, DN_V_SIZE, DN_HEADS, DN_HEADS};
                for (int i = 0, col = 0; i < 4; col += rows[i], ++i)
                    Q35_TRY(gemm_bf16(a.normalized, HIDDEN, (const bf16*)L.p[slot[i]], rows[i], a.proj_buf + col, ldp, nullptr, 0, S, rows[i], HIDDEN, 0, 0, stream));
            }
            Q35_CUDA_OK(pdl_launch(pf_dn_prep_kernel, (S * DN_HEADS + DN_PREP_WARPS - 1) / DN_PREP_WARPS, 32 * DN_PREP_WARPS, 0, stream, a.proj_buf, ldp, (const bf16*)L.p[DN_CONV], (const bf16*)L.p[DN_ALOG],
                                                                      (const bf16*)L.p[DN_DTBIAS], a.proj_buf2, a.beta_buf, a.alpha_buf,
                                                                      a.conv_bufs + (size_t)i_dn * DN_CONV_CH * 4, S));
            Q35_CUDA_OK(pdl_launch(pf_dn_chunk_local_kernel, dim3(nchunks, DN_HEADS), CL_THREADS, CHUNK_LOCAL_SMEM, stream, a.proj_buf2, a.beta_buf, a.alpha_buf, scratch, S, nchunks));
            Q35_CUDA_OK(pdl_launch(pf_dn_chunk_scan_kernel, dim3(DN_HEADS, DN_V / SCAN_VW), SCAN_THREADS, CHUNK_SCAN_SMEM, stream, 
                scratch, a.dn_out_buf, a.dn_states + (size_t)i_dn * DN_HEADS * DN_V * DN_K, S, nchunks, err_word));
            Q35_CUDA_OK(pdl_launch(pf_gated_norm_kernel<false>, (S * DN_HEADS + 15) / 16, 256, 0, stream, a.dn_out_buf, a.proj_buf, ldp, (const bf16*)L.p[DN_NORM], a.attn_buf, S));
            g_launches.fetch_add(4);
            w_out = (const bf16*)L.p[DN_OUT]; w_post = (const bf16*)L.p[DN_POST_NORM]; w_down = (const bf16*)L.p[DN_DOWN];
            ++i_dn;
        } else {
            const int ldp = FA_PROJ_ROWS;
            if (fp4) {
                Q35_TRY(gemm_nvfp4(act_packed, act_scales, S, F->proj_packed, F->proj_scales, FA_PROJ_ROWS, FA_PROJ_ROWS, HIDDEN, 1.0f, a.proj_buf, ldp, 0,
                                   nullptr, 0, stream));
            } else if (F) {
                Q35_TRY(gemm_bf16(a.normalized, HIDDEN, (const bf16*)F->proj_weight, FA_PROJ_ROWS, a.proj_buf, ldp, nullptr, 0, S, FA_PROJ_ROWS, HIDDEN, 0, 0, stream));
            } else {
                const int slot[3] = {FA_Q, FA_K, FA_V}, rows[3] = {FA_QPROJ, FA_KV_SIZE, FA_KV_SIZE};
                for (int i = 0, col = 0; i < 3; col += rows[i], ++i)
                    Q35_TRY(gemm_bf16(a.normalized, HIDDEN, (const bf16*)L.p[slot[i]], rows[i], a.proj_buf + col, ldp, nullptr, 0, S, rows[i], HIDDEN, 0, 0, stream));
            }
            bf16* kc = a.k_cache + (size_t)i_fa * FA_KV_HEADS * a.max_seq_len * FA_HEAD_DIM;
            bf16* vc = a.v_cache + (size_t)i_fa * FA_KV_HEADS * a.max_seq_len * FA_HEAD_DIM;
            Q35_CUDA_OK(pdl_launch(pf_qk_norm_rope_kernel, (S * 12 + 7) / 8, 256, 0, stream, a.proj_buf, ldp, (const bf16*)L.p[FA_QNORM], (const bf16*)L.p[FA_KNORM], rt,
                                                                         a.proj_buf2, kc, vc, S, a.max_seq_len));
            Q35_TRY(attention_prefill_tcgen05(a.proj_buf2, kc, vc, a.proj_buf, ldp, a.attn_buf, vt_scratch, S, a.max_seq_len, stream));
            g_launches.fetch_add(1);
            w_out = (const bf16*)L.p[FA_O]; w_post = (const bf16*)L.p[FA_POST_NORM]; w_down = (const bf16*)L.p[FA_DOWN];
            ++i_fa;
        }
        // output projection + residual -> residual buffer holds the hidden state after the mixer
        Q35_TRY(gemm_bf16(a.attn_buf, 2048, w_out, HIDDEN, a.residual, HIDDEN, layer_in, HIDDEN, S, HIDDEN, 2048, 1, 0, stream));
        Q35_CUDA_OK(pdl_launch(pf_rmsnorm_kernel<false>, fp4 ? s_pad : S, 128, 0, stream, nullptr, nullptr, a.residual, w_post, nullptr, fp4 ? (bf16*)nullptr : a.normalized, S,
                                                 fp4 ? (uint8_t*)act_packed : (uint8_t*)nullptr, fp4 ? (uint8_t*)act_scales : (uint8_t*)nullptr));
        g_launches.fetch_add(1);
        if (fp4) {
            // [gate | up] rows of one block-scaled GEMM into proj_buf ([S, 7168]; the projection buffer is free again), then SiLU * up
            Q35_TRY(gemm_nvfp4(act_packed, act_scales, S, F->gate_up_packed, F->gate_up_scales, 2 * INTER, 2 * INTER, HIDDEN, 1.0f, a.proj_buf, 2 * INTER, 0,
                               nullptr, 0, stream));
            Q35_CUDA_OK(pdl_launch(pf_silu_mul_rows_kernel, (S * (INTER / 8) + 255) / 256, 256, 0, stream, (const bf16*)a.proj_buf, a.mlp_buf, S));
            g_launches.fetch_add(1);
        } else if (F) {
            Q35_TRY(gemm_bf16(a.normalized, HIDDEN, (const bf16*)F->gate_up_weight, 2 * INTER, a.mlp_buf, INTER, nullptr, 0, S, INTER, HIDDEN, 2, INTER, stream));
        } else {
            // the projection buffers are free again here: gate -> proj_buf, up -> proj_buf2 (both [S, 3584])
            const bool dn = L.type == 0;
            Q35_TRY(gemm_bf16(a.normalized, HIDDEN, (const bf16*)L.p[dn ? (int)DN_GATE : (int)FA_GATE], INTER, a.proj_buf, INTER, nullptr, 0, S, INTER, HIDDEN, 0, 0, stream));
            Q35_TRY(gemm_bf16(a.normalized, HIDDEN, (const bf16*)L.p[dn ? (int)DN_UP : (int)FA_UP], INTER, a.proj_buf2, INTER, nullptr, 0, S, INTER, HIDDEN, 0, 0, stream));
            const int n8 = S * INTER / 8;
            Q35_CUDA_OK(pdl_launch(pf_silu_mul_kernel, (n8 + 255) / 256, 256, 0, stream, (const bf16*)a.proj_buf, (const bf16*)a.proj_buf2, a.mlp_buf, n8));
            g_launches.fetch_add(1);
        }
        Q35_TRY(gemm_bf16(a.mlp_buf, INTER, w_down, HIDDEN, a.hidden, HIDDEN, a.residual, HIDDEN, S, HIDDEN, INTER, 1, 0, stream));
        if (a.dbg_hidden)
            Q35_CUDA_OK(cudaMemcpyAsync(a.dbg_hidden + (size_t)layer * HIDDEN, a.hidden + (size_t)(S - 1) * HIDDEN, HIDDEN * sizeof(bf16), cudaMemcpyDeviceToDevice, stream));
    }
    // last token: final norm, LM head, arg-max
    const bf16* last = a.hidden + (size_t)(S - 1) * HIDDEN;
    if (a.hidden_out) Q35_CUDA_OK(cudaMemcpyAsync(a.hidden_out, last, HIDDEN * sizeof(bf16), cudaMemcpyDeviceToDevice, stream));
    Q35_CUDA_OK(pdl_launch(pf_rmsnorm_kernel<false>, a.lm_packed ? 128 : 1, 128, 0, stream, nullptr, nullptr, last, a.final_norm, nullptr, a.final_normed, 1,
                                             a.lm_packed ? (uint8_t*)act_packed : (uint8_t*)nullptr, a.lm_packed ? (uint8_t*)act_scales : (uint8_t*)nullptr));
    const int lm_blocks = 592;
    if (a.lm_packed) {
        // the reference's FP4 head (kernel_gb10_nvfp4.cu:1945-1997): the normed hidden row is quantised to NVFP4 as well and the
        // block-scaled tensor-core GEMM gives the logits, rounded once to bf16; arg-max with the lowest index among ties
        Q35_TRY(gemm_nvfp4(act_packed, act_scales, 1, a.lm_packed, a.lm_scales, VOCAB, VOCAB, HIDDEN, 1.0f, lm_logits, VOCAB, 0, nullptr, 0, stream));
        Q35_CUDA_OK(pdl_launch(pf_argmax_row_kernel, 1, 1024, 0, stream, (const bf16*)lm_logits, a.out_token, a.logits_out));
        g_launches.fetch_add(2);
    } else {
        Q35_CUDA_OK(pdl_launch(pf_lm_head_kernel, lm_blocks, 256, 0, stream, a.final_normed, a.lm_head, a.lm_bmv, a.lm_bmi, a.logits_out));
        Q35_CUDA_OK(pdl_launch(pf_lm_reduce_kernel, 1, 32, 0, stream, a.lm_bmv, a.lm_bmi, lm_blocks, a.out_token));
        g_launches.fetch_add(3);
    }
    Q35_CUDA_OK(cudaGetLastError());
    return QWEN35_OK;
}

// The layer tables live in device memory (the reference's packed blobs).  As in the reference (prefill.cu:1179-1195)
// they are read back once per distinct pair of table pointers and kept on the host, so later calls neither
// synchronise nor allocate (a prefill can then be captured in a CUDA graph).  A caller that frees its tables and
// packs new ones can get the same device address back with different contents: it calls
// qwen35_b200_forget_tables() after re-packing (both Python hosts do so whenever a table tensor they have not seen
// appears).  The caller receives a COPY made under the lock, so an entry that is evicted or forgotten while another
// thread is still launching from its copy cannot dangle.  dev_fused may be null (launch_prefill_bf16_mega has none).
static HostTables g_tables[8];
static int g_tables_n = 0, g_tables_next = 0;
static std::mutex g_tables_mu;

bool host_layer_tables(const void* dev_layers, const void* dev_fused, HostTables* out) {
    std::lock_guard<std::mutex> lk(g_tables_mu);
    for (int i = 0; i < g_tables_n; ++i)
        if (g_tables[i].dev_layers == dev_layers && g_tables[i].dev_fused == dev_fused) { *out = g_tables[i]; return true; }
    HostTables t = {};
    t.dev_layers = dev_layers; t.dev_fused = dev_fused;
    if (cudaMemcpy(t.layers, dev_layers, sizeof(t.layers), cudaMemcpyDeviceToHost) != cudaSuccess ||
        (dev_fused && cudaMemcpy(t.fused, dev_fused, sizeof(t.fused), cudaMemcpyDeviceToHost) != cudaSuccess)) {
        set_error("reading the layer tables failed: %s", cudaGetErrorString(cudaGetLastError()));
        return false;
    }
    // a full cache evicts its entries in turn
    const int slot = g_tables_n < 8 ? g_tables_n++ : (g_tables_next++ & 7);
    g_tables[slot] = t;
    *out = t;
    return true;
}

void forget_layer_tables() {
    std::lock_guard<std::mutex> lk(g_tables_mu);
    g_tables_n = 0;
    g_tables_next = 0;
}

}  // namespace q35

extern "C" void qwen35_b200_forget_tables(void) { q35::forget_layer_tables(); }

extern "C" int qwen35_b200_prefill_bf16(const Qwen35PrefillArgs* in, qwen35_stream_t stream) {
    using namespace q35;
    if (!in) { set_error("null args"); return QWEN35_ERR_BAD_ARG; }
    if (in->seq_len <= 0 || in->seq_len > in->max_seq_len || in->seq_len > ATT_PF_MAX_S) {
        set_error("seq_len %d out of range (max_seq_len %d, library limit %d)", in->seq_len, in->max_seq_len, ATT_PF_MAX_S);
        return QWEN35_ERR_BAD_ARG;
    }
    if (!in->token_ids || !in->embed_weight || !in->layer_weights || !in->hidden || !in->proj_buf) {
        set_error("null tensor pointer");
        return QWEN35_ERR_BAD_ARG;
    }
    HostTables tables;
    if (!host_layer_tables(in->layer_weights, in->fused_layer_weights, &tables)) return QWEN35_ERR_CUDA;
    PrefillArgs a = {};
    a.token_ids = in->token_ids; a.S = in->seq_len; a.out_token = in->out_token;
    a.embed = (const bf16*)in->embed_weight; a.layers_host = tables.layers; a.fused_host = in->fused_layer_weights ? tables.fused : nullptr;
    a.final_norm = (const bf16*)in->final_norm_weight; a.lm_head = (const bf16*)in->lm_head_weight;
    a.k_cache = (bf16*)in->fa_k_cache; a.v_cache = (bf16*)in->fa_v_cache; a.dn_states = (float*)in->dn_states; a.conv_bufs = (float*)in->conv_bufs;
    a.hidden = (bf16*)in->hidden; a.residual = (bf16*)in->residual; a.normalized = (bf16*)in->normalized;
    a.proj_buf = (bf16*)in->proj_buf; a.proj_buf2 = (bf16*)in->proj_buf2; a.attn_buf = (bf16*)in->attn_buf; a.mlp_buf = (bf16*)in->mlp_buf;
    a.dn_out_buf = (bf16*)in->dn_out_buf; a.beta_buf = (float*)in->beta_buf; a.alpha_buf = (float*)in->alpha_buf;
    a.final_normed = (bf16*)in->final_normed; a.hidden_out = (bf16*)in->hidden_bf16_out;
    a.lm_bmv = (float*)in->lm_bmv; a.lm_bmi = (int*)in->lm_bmi; a.logits_out = in->logits_out;
    a.lm_packed = in->lm_head_weight_packed; a.lm_scales = in->lm_head_scales;
    a.max_seq_len = in->max_seq_len;
    a.dbg_teacher = (const bf16*)in->dbg_teacher; a.dbg_hidden = (bf16*)in->dbg_hidden;
    a.n_layers = in->dbg_num_layers > 0 ? in->dbg_num_layers : NUM_LAYERS;
    return prefill_impl(a, (cudaStream_t)stream);
}

extern "C" int launch_prefill_bf16(
    const int* token_ids, int seq_len, int* output_token,
    const void* embed_weight, const LayerWeights* layers, const void* fused_layers,
    const void* final_norm_w, const void* lm_head_w,
    void* fa_k_cache, void* fa_v_cache, void* dn_states, void* conv_bufs,
    void* hidden, void* residual, void* normalized,
    void* proj_buf, void* proj_buf2, void* /*proj_buf_half*/, void* /*proj_act_packed*/, void* /*proj_act_scales*/,
    void* attn_buf, void* mlp_buf, void* dn_out_buf, void* beta_buf, void* alpha_buf,
    void* final_normed, void* hidden_bf16_out, void* lm_bmv, void* lm_bmi, qwen35_stream_t stream) {
    Qwen35PrefillArgs a = {};
    a.token_ids = token_ids; a.seq_len = seq_len; a.out_token = output_token;
    a.embed_weight = embed_weight; a.layer_weights = layers; a.fused_layer_weights = fused_layers;
    a.final_norm_weight = final_norm_w; a.lm_head_weight = lm_head_w;
    a.fa_k_cache = fa_k_cache; a.fa_v_cache = fa_v_cache; a.dn_states = dn_states; a.conv_bufs = conv_bufs;
    a.hidden = hidden; a.residual = residual; a.normalized = normalized; a.proj_buf = proj_buf; a.proj_buf2 = proj_buf2;
    a.attn_buf = attn_buf; a.mlp_buf = mlp_buf; a.dn_out_buf = dn_out_buf; a.beta_buf = beta_buf; a.alpha_buf = alpha_buf;
    a.final_normed = final_normed; a.hidden_bf16_out = hidden_bf16_out; a.lm_bmv = lm_bmv; a.lm_bmi = lm_bmi;
    a.max_seq_len = 2048;       // the reference's fixed cache length (prefill.cu:1203, 1394)
    return qwen35_b200_prefill_bf16(&a, stream);
}

// Replaces launch_prefill_bf16_nvfp4_lm (torch_bindings.cpp:337-352; prefill.cu:1499-1534): the bf16 prefill body with the
// NVFP4 LM head for the last token.
extern "C" int launch_prefill_bf16_nvfp4_lm(
    const int* token_ids, int seq_len, int* output_token,
    const void* embed_weight, const LayerWeights* layers, const void* fused_layers,
    const void* final_norm_w, const void* lm_head_w, const void* lm_head_weight_packed, const void* lm_head_scales,
    void* fa_k_cache, void* fa_v_cache, void* dn_states, void* conv_bufs,
    void* hidden, void* residual, void* normalized,
    void* proj_buf, void* proj_buf2, void* /*proj_buf_half*/, void* /*proj_act_packed*/, void* /*proj_act_scales*/,
    void* attn_buf, void* mlp_buf, void* dn_out_buf, void* beta_buf, void* alpha_buf,
    void* final_normed, void* hidden_bf16_out, void* lm_bmv, void* lm_bmi,
    void* /*lm_hidden_bf16*/, void* /*lm_hidden_packed*/, void* /*lm_hidden_scales*/, void* /*lm_logits_f16*/, qwen35_stream_t stream) {
    Qwen35PrefillArgs a = {};
    a.token_ids = token_ids; a.seq_len = seq_len; a.out_token = output_token;
    a.embed_weight = embed_weight; a.layer_weights = layers; a.fused_layer_weights = fused_layers;
    a.final_norm_weight = final_norm_w; a.lm_head_weight = lm_head_w;
    a.lm_head_weight_packed = lm_head_weight_packed; a.lm_head_scales = lm_head_scales;
    a.fa_k_cache = fa_k_cache; a.fa_v_cache = fa_v_cache; a.dn_states = dn_states; a.conv_bufs = conv_bufs;
    a.hidden = hidden; a.residual = residual; a.normalized = normalized; a.proj_buf = proj_buf; a.proj_buf2 = proj_buf2;
    a.attn_buf = attn_buf; a.mlp_buf = mlp_buf; a.dn_out_buf = dn_out_buf; a.beta_buf = beta_buf; a.alpha_buf = alpha_buf;
    a.final_normed = final_normed; a.hidden_bf16_out = hidden_bf16_out; a.lm_bmv = lm_bmv; a.lm_bmi = lm_bmi;
    a.max_seq_len = 2048;
    return qwen35_b200_prefill_bf16(&a, stream);
}

// Replaces launch_prefill_bf16_mega (torch_bindings.cpp:354-364; prefill_megakernel.cu:840-1078), the reference's
// single-dispatch prompt pass.  Same results as launch_prefill_bf16; it has no fused-weight table, so each matrix of the
// layer records runs as its own tensor-core GEMM (the reference's version does the same work from one persistent grid at
// 58.6 ms for 520 tokens; this one is a stream of launches chained by programmatic dependent launch).
extern "C" int launch_prefill_bf16_mega(
    const int* token_ids, int seq_len, int* output_token,
    const void* embed_weight, const LayerWeights* layers,
    const void* final_norm_w, const void* lm_head_w,
    void* fa_k_cache, void* fa_v_cache, void* dn_states, void* conv_bufs,
    void* hidden, void* residual, void* normalized,
    void* proj_buf, void* proj_buf2, void* attn_buf, void* mlp_buf,
    void* dn_out_buf, void* beta_buf, void* alpha_buf,
    void* final_normed, void* hidden_bf16_out, void* lm_bmv, void* lm_bmi, qwen35_stream_t stream) {
    Qwen35PrefillArgs a = {};
    a.token_ids = token_ids; a.seq_len = seq_len; a.out_token = output_token;
    a.embed_weight = embed_weight; a.layer_weights = layers; a.fused_layer_weights = nullptr;
    a.final_norm_weight = final_norm_w; a.lm_head_weight = lm_head_w;
    a.fa_k_cache = fa_k_cache; a.fa_v_cache = fa_v_cache; a.dn_states = dn_states; a.conv_bufs = conv_bufs;
    a.hidden = hidden; a.residual = residual; a.normalized = normalized; a.proj_buf = proj_buf; a.proj_buf2 = proj_buf2;
    a.attn_buf = attn_buf; a.mlp_buf = mlp_buf; a.dn_out_buf = dn_out_buf; a.beta_buf = beta_buf; a.alpha_buf = alpha_buf;
    a.final_normed = final_normed; a.hidden_bf16_out = hidden_bf16_out; a.lm_bmv = lm_bmv; a.lm_bmi = lm_bmi;
    a.max_seq_len = 2048;       // MAX_SEQ of the reference's megakernel (prefill_megakernel.cu:37)
    return qwen35_b200_prefill_bf16(&a, stream);
}
