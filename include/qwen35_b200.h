/*
 * C ABI of libqwen35_b200.so -- the B200 (sm_100a) implementation of the Qwen3.5 hybrid
 * forward path behind lucebox-hub's torch-extension boundary.
 *
 * Every `launch_*` entry point has the argument list of the function of the same name that the
 * reference's binding layer declares and calls (models/qwen35_0p8b/torch_bindings.cpp); the
 * citation beside each declaration gives the lines.  Differences from the reference, all
 * additive:
 *   - every function returns an int status (0 = enqueued / ok) instead of void;
 *   - `max_seq_len` is honoured (the reference hard-codes 2048 in its prefill);
 *   - scratch arguments the reference kernels needed are accepted and ignored -- the library
 *     keeps one private workspace per device, allocated on the first call on that device
 *     (make that first call outside CUDA-graph capture).
 * All pointers are device pointers unless stated otherwise.  Work is enqueued on `stream`; no
 * entry point synchronises except qwen35_b200_status().
 */
#ifndef QWEN35_B200_H
#define QWEN35_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* qwen35_stream_t; /* == cudaStream_t */

/* Layer pointer records, layout of the reference (kernel.cu:77-115, torch_bindings.cpp:25-45). */
typedef struct {
    int layer_type;      /* 0 = DeltaNet (14 pointers), 1 = full attention (11 pointers) */
    int _pad[3];
    void* ptrs[14];      /* bf16 tensors in the order of models/qwen35_0p8b/model.py:342-380 */
} LayerWeights;

enum {
    QWEN35_OK = 0,
    QWEN35_ERR_BARRIER_TIMEOUT = 1, /* a bounded device-side wait ran out; state is undefined */
    QWEN35_ERR_BAD_ARG = 2,
    QWEN35_ERR_CUDA = 3,
    QWEN35_ERR_UNSUPPORTED = 4
};

/* Replaces launch_decode (torch_bindings.cpp:47-60; kernel.cu:910-1020): one greedy decode step.
 * Reads embed[input_token_id], runs 24 layers at `position`, appends K/V, updates the DeltaNet
 * and conv state in place, writes arg-max(logits) to output_token_id[0].  The arg-max is taken
 * over bf16-rounded logits and returns the lowest index among equal maxima. */
int launch_decode(
    int input_token_id, int* output_token_id,
    const void* embed_weight, const LayerWeights* layer_weights,
    const void* final_norm_weight, const void* lm_head_weight,
    void* fa_k_cache, void* fa_v_cache,
    void* dn_states, void* conv_bufs,
    void* hidden_buffer, void* g_activations, void* g_residual,
    void* g_qkv_scratch, void* g_kv_scratch, void* g_attn_out,
    void* g_mlp_inter, void* g_z_scratch, void* g_beta_scratch,
    void* g_alpha_scratch, void* g_normalized,
    unsigned int* barrier_counter, unsigned int* barrier_generation,
    float* block_max_vals, int* block_max_idxs,
    unsigned int* lm_sync_counter,
    int position, int max_seq_len, qwen35_stream_t stream);

/* Extended decode / token-serial prefill.  No counterpart in the reference's BF16 path (its NVFP4
 * path has the same idea in launch_decode_many_nvfp4, torch_bindings.cpp:87-102): runs `n_steps`
 * steps in one launch, feeding each arg-max back on the device. */
typedef struct {
    const void* embed_weight;
    const void* layer_weights; /* LayerWeights records, or LayerWeightsNVFP4 records for the NVFP4 entry point */
    const void* final_norm_weight;
    const void* lm_head_weight;
    void* fa_k_cache;          /* bf16 [6][2][max_seq_len][256] */
    void* fa_v_cache;
    void* dn_states;           /* f32 [18][16][128 v][128 k] */
    void* conv_bufs;           /* f32 [18][6144][4], newest input last */
    const int* token_in;       /* device int: first input token; NULL -> token_imm */
    int token_imm;
    const int* forced_ids;     /* optional device [n_steps]: input of every step (prompt / teacher forcing) */
    int* out_token;            /* optional device [1]: arg-max of the last step */
    int* out_tokens;           /* optional device [n_steps]: arg-max of every step that ran the LM head */
    float* logits_out;         /* optional device f32 [248320]: bf16-rounded logits of the last step */
    void* hidden_out;          /* optional device bf16 [1024]: last layer output of the last step */
    void* dbg_hidden;          /* optional device bf16 [24][1024]: every layer's output, last step */
    const void* dbg_teacher;   /* optional device bf16 [24][1024]: layer l>0 reads row l as its input (layer-level parity tests) */
    int position;
    int max_seq_len;
    int n_steps;
    int lm_last_only;          /* 1 = run the LM head only after the last step */
    int dbg_num_layers;        /* 0 = all 24; N>0 stops after N layers (debug) */
    unsigned long long* dbg_time; /* optional device u64 [grid][25][12]: per-stage time stamps of every CTA, last step */
    int dbg_time_cta;             /* -2: stamps are SM cycle counts (clock64, exact within a CTA); otherwise %globaltimer ns */
} Qwen35DecodeArgs;

int qwen35_b200_decode_steps(const Qwen35DecodeArgs* args, qwen35_stream_t stream);

/* Replaces launch_prefill_bf16 (torch_bindings.cpp:323-335; prefill.cu:1158-1497): batched prefill of
 * `seq_len` prompt tokens from a zeroed state.  Fills the KV cache rows [0, seq_len), the DeltaNet states and
 * conv windows, writes the last token's hidden state to hidden_bf16_out and arg-max(logits) to output_token.
 * Scratch buffers have the sizes the reference's Decoder allocates (model.py:569-602); proj_buf_half,
 * proj_act_packed and proj_act_scales belong to the reference's NVFP4 option and are ignored.  `fused_layers`
 * is the device table of PrefillFusedLayerWeights records (6 pointers per layer, prefill.cu:66-73).  The cache
 * length is the reference's fixed 2048; use qwen35_b200_prefill_bf16 for other lengths. */
int launch_prefill_bf16(
    const int* token_ids, int seq_len, int* output_token,
    const void* embed_weight, const LayerWeights* layers, const void* fused_layers,
    const void* final_norm_w, const void* lm_head_w,
    void* fa_k_cache, void* fa_v_cache, void* dn_states, void* conv_bufs,
    void* hidden, void* residual, void* normalized,
    void* proj_buf, void* proj_buf2, void* proj_buf_half, void* proj_act_packed, void* proj_act_scales,
    void* attn_buf, void* mlp_buf, void* dn_out_buf, void* beta_buf, void* alpha_buf,
    void* final_normed, void* hidden_bf16_out, void* lm_bmv, void* lm_bmi, qwen35_stream_t stream);

/* Replaces launch_prefill_bf16_nvfp4_lm (torch_bindings.cpp:337-352): the same prefill with the last token's LM head read
 * from the NVFP4 tensor-core layout.  The reference's activation quantisation buffers (lm_hidden_*, lm_logits_f16) are ignored. */
int launch_prefill_bf16_nvfp4_lm(
    const int* token_ids, int seq_len, int* output_token,
    const void* embed_weight, const LayerWeights* layers, const void* fused_layers,
    const void* final_norm_w, const void* lm_head_w, const void* lm_head_weight_packed, const void* lm_head_scales,
    void* fa_k_cache, void* fa_v_cache, void* dn_states, void* conv_bufs,
    void* hidden, void* residual, void* normalized,
    void* proj_buf, void* proj_buf2, void* proj_buf_half, void* proj_act_packed, void* proj_act_scales,
    void* attn_buf, void* mlp_buf, void* dn_out_buf, void* beta_buf, void* alpha_buf,
    void* final_normed, void* hidden_bf16_out, void* lm_bmv, void* lm_bmi,
    void* lm_hidden_bf16, void* lm_hidden_packed, void* lm_hidden_scales, void* lm_logits_f16, qwen35_stream_t stream);

/* Replaces launch_prefill_bf16_mega (torch_bindings.cpp:354-364; prefill_megakernel.cu:840-1078), the reference's single-
 * dispatch prompt pass: same inputs and results as launch_prefill_bf16 without the fused-weight table.  Each matrix of the
 * layer records runs as its own tensor-core GEMM into the column blocks of proj_buf; SiLU(gate)*up is a kernel of its own
 * (gate in proj_buf, up in proj_buf2).  Cache length 2048 (MAX_SEQ, prefill_megakernel.cu:37). */
int launch_prefill_bf16_mega(
    const int* token_ids, int seq_len, int* output_token,
    const void* embed_weight, const LayerWeights* layers,
    const void* final_norm_w, const void* lm_head_w,
    void* fa_k_cache, void* fa_v_cache, void* dn_states, void* conv_bufs,
    void* hidden, void* residual, void* normalized,
    void* proj_buf, void* proj_buf2, void* attn_buf, void* mlp_buf,
    void* dn_out_buf, void* beta_buf, void* alpha_buf,
    void* final_normed, void* hidden_bf16_out, void* lm_bmv, void* lm_bmi, qwen35_stream_t stream);

/* The same with an explicit cache length, optional logits and a layer limit for tests.  fused_layer_weights may be NULL:
 * the pass then takes every matrix from layer_weights (the launch_prefill_bf16_mega form). */
typedef struct {
    const int* token_ids; int seq_len; int* out_token;
    const void* embed_weight; const LayerWeights* layer_weights; const void* fused_layer_weights;
    const void* final_norm_weight; const void* lm_head_weight;
    void* fa_k_cache; void* fa_v_cache; void* dn_states; void* conv_bufs;
    void* hidden;        /* bf16 [S,1024]: layer input / output */
    void* residual;      /* bf16 [S,1024]: hidden after the mixer residual */
    void* normalized;    /* bf16 [S,1024] */
    void* proj_buf;      /* bf16 [S,8320] */
    void* proj_buf2;     /* bf16 [S,6144] */
    void* attn_buf;      /* bf16 [S,2048] */
    void* mlp_buf;       /* bf16 [S,3584] */
    void* dn_out_buf;    /* bf16 [S,2048] */
    void* beta_buf;      /* f32 [S,16] */
    void* alpha_buf;     /* f32 [S,16] */
    void* final_normed;  /* bf16 [1024] */
    void* hidden_bf16_out; /* bf16 [1024] */
    void* lm_bmv;        /* f32 [1024] */
    void* lm_bmi;        /* i32 [1024] */
    float* logits_out;   /* optional f32 [248320] */
    int max_seq_len;
    int dbg_num_layers;  /* 0 = all */
    const void* lm_head_weight_packed; /* optional: NVFP4 LM head (tensor-core layout) used for the last token */
    const void* lm_head_scales;
    const void* dbg_teacher; /* optional bf16 [24][seq_len][1024]: layer l>0 reads row block l as its input (layer-level parity tests) */
    void* dbg_hidden;        /* optional bf16 [24][1024]: every layer's output at the last position */
} Qwen35PrefillArgs;
int qwen35_b200_prefill_bf16(const Qwen35PrefillArgs* args, qwen35_stream_t stream);

/* NVFP4 decode.  Replaces launch_decode_nvfp4 (torch_bindings.cpp:62-77; kernel_gb10_nvfp4.cu:1999-2183) and
 * launch_decode_many_nvfp4 (torch_bindings.cpp:87-102; kernel_gb10_nvfp4.cu:2185-2250).  layer_weights is the device
 * table of LayerWeightsNVFP4 records {int type; int group_size; int pad[2]; void* ptrs[24]} (slot order of
 * model.py:248-284: packed nibbles + fp16 group scales per quantised matrix, group_size 32); the LM head is in
 * the tensor-core layout (packed + swizzled E4M3 block scales).  Weights are dequantised in registers and
 * multiplied with the bf16 activations in f32; the reference's FP4 quantisation of the LM-head activation is
 * not reproduced.  The input token is read from device memory so steps chain without a host round trip;
 * launch_decode_many_nvfp4 runs `steps` steps in one launch, token_buffer[0] in/out.  The lm_hidden_* /
 * lm_logits_f16 and scratch arguments of the reference are accepted and ignored. */
int launch_decode_nvfp4(
    const int* input_token_ptr, int* output_token_id, const void* embed_weight, const void* layer_weights,
    const void* final_norm_weight, const void* lm_head_weight_packed, const void* lm_head_scales,
    void* lm_hidden_bf16, void* lm_hidden_packed, void* lm_hidden_scales, void* lm_logits_f16,
    void* fa_k_cache, void* fa_v_cache, void* dn_states, void* conv_bufs, void* hidden_buffer,
    void* g_activations, void* g_residual, void* g_qkv_scratch, void* g_kv_scratch, void* g_attn_out,
    void* g_mlp_inter, void* g_z_scratch, void* g_beta_scratch, void* g_alpha_scratch, void* g_normalized,
    unsigned int* barrier_counter, unsigned int* barrier_generation, float* block_max_vals, int* block_max_idxs,
    unsigned int* lm_sync_counter, int position, int max_seq_len, int group_size, qwen35_stream_t stream);
int launch_decode_many_nvfp4(
    int* token_buffer, int* output_tokens, int steps, const void* embed_weight, const void* layer_weights,
    const void* final_norm_weight, const void* lm_head_weight_packed, const void* lm_head_scales,
    void* lm_hidden_bf16, void* lm_hidden_packed, void* lm_hidden_scales, void* lm_logits_f16,
    void* fa_k_cache, void* fa_v_cache, void* dn_states, void* conv_bufs, void* hidden_buffer,
    void* g_activations, void* g_residual, void* g_qkv_scratch, void* g_kv_scratch, void* g_attn_out,
    void* g_mlp_inter, void* g_z_scratch, void* g_beta_scratch, void* g_alpha_scratch, void* g_normalized,
    unsigned int* barrier_counter, unsigned int* barrier_generation, float* block_max_vals, int* block_max_idxs,
    unsigned int* lm_sync_counter, int position, int max_seq_len, int group_size, qwen35_stream_t stream);
/* Replaces launch_prefill_megakernel_nvfp4 (torch_bindings.cpp:104-119; kernel_gb10_nvfp4.cu:1659-1755, 2119-2183): the
 * single-dispatch prompt pass of the NVFP4 path.  Token-serial like the reference's: the decode megakernel runs the seq_len
 * prompt tokens from position 0 in one launch, the LM head after the last; output_token_id[0] = the first generated token. */
int launch_prefill_megakernel_nvfp4(
    const int* token_ids, int seq_len, int* output_token_id, const void* embed_weight, const void* layer_weights,
    const void* final_norm_weight, const void* lm_head_weight_packed, const void* lm_head_scales,
    void* lm_hidden_bf16, void* lm_hidden_packed, void* lm_hidden_scales, void* lm_logits_f16,
    void* fa_k_cache, void* fa_v_cache, void* dn_states, void* conv_bufs, void* hidden_buffer,
    void* g_activations, void* g_residual, void* g_qkv_scratch, void* g_kv_scratch, void* g_attn_out,
    void* g_mlp_inter, void* g_z_scratch, void* g_beta_scratch, void* g_alpha_scratch, void* g_normalized,
    unsigned int* barrier_counter, unsigned int* barrier_generation, float* block_max_vals, int* block_max_idxs,
    unsigned int* lm_sync_counter, int max_seq_len, int group_size, qwen35_stream_t stream);
/* qwen35_b200_decode_steps for the NVFP4 format (logits, teacher forcing, debug outputs). */
int qwen35_b200_decode_steps_nvfp4(const Qwen35DecodeArgs* args, const void* lm_head_scales, qwen35_stream_t stream);

/* Replaces launch_quantize_nvfp4_out (torch_bindings.cpp:79-81; kernel_gb10_nvfp4.cu:1757-1876): pack a bf16
 * matrix [rows, cols] into the decode-body NVFP4 layout: packed uint8 [rows, cols/2] (low nibble = even
 * element) and fp16 scales [rows, cols/group_size]. */
int launch_quantize_nvfp4_out(const void* weight, int rows, int cols, int group_size, void* packed_out, void* scales_out,
                              qwen35_stream_t stream);

/* Replaces launch_quantize_nvfp4_lm_out (torch_bindings.cpp:83-85; kernel_gb10_nvfp4.cu:1366-1430, 1878-1892):
 * the tensor-core layout: 16-element blocks, UE4M3 block scales in 128x4 swizzled tiles
 * (byte = tile*512 + (row%32)*16 + ((row%128)/32)*4 + block%4, tile = (row/128)*(cols/64) + block/4), per-tensor
 * scale 1.0.  rows must be a multiple of 128 and cols a multiple of 64. */
int launch_quantize_nvfp4_lm_out(const void* weight, int rows, int cols, void* packed_out, void* scales_out, qwen35_stream_t stream);

/* Batched greedy decode (no counterpart in the reference, which is batch-1 only: README.md:167): `batch`
 * independent sequences advance one token.  Each sequence follows the bs=1 arithmetic of launch_decode.
 *   tokens_in / tokens_out  int32 [batch]            positions  int32 [batch] tokens already cached per sequence
 *   k_pages / v_pages       bf16 [6][num_pages][2][64][256], addressed through block_table int32 [batch][max_pages]
 *   dn_states f32 [batch][18][16][128][128]          conv_bufs f32 [batch][18][6144][4]
 * max_ctx bounds positions+1 (<= 8192).  advance_positions != 0 increments positions[] on the device after the
 * step, so steps chain without host work.  Weights are the bf16 tables of launch_prefill_bf16.
 * layer_weights_host / fused_layer_weights_host: optional host copies of the two device tables (same bytes).  With
 * them no call ever synchronises; without them the first call with a new pair of device tables reads them back
 * (see qwen35_b200_forget_tables). */
typedef struct {
    int batch; int max_ctx; int num_pages; int max_pages;
    const int* tokens_in; int* tokens_out; int* positions; const int* block_table;
    const void* embed_weight; const LayerWeights* layer_weights; const void* fused_layer_weights;
    const void* final_norm_weight; const void* lm_head_weight;
    void* k_pages; void* v_pages; void* dn_states; void* conv_bufs;
    void* logits_out;          /* optional bf16 [batch][248320] */
    void* dbg_hidden;          /* optional bf16 [24][batch][1024]: every layer's output */
    const void* dbg_teacher;   /* optional bf16 [24][batch][1024]: layer l>0 reads row block l as its input */
    int advance_positions;
    int dbg_num_layers;
    const void* layer_weights_host; const void* fused_layer_weights_host;
    void* scratch; size_t scratch_bytes;   /* optional caller-owned scratch (256-byte aligned, >= qwen35_b200_batched_scratch_bytes):
                                              required when two calls run concurrently on two streams; null = the library's own */
} Qwen35BatchedArgs;
int qwen35_b200_decode_batched(const Qwen35BatchedArgs* args, qwen35_stream_t stream);
size_t qwen35_b200_batched_scratch_bytes(int batch, int max_ctx);

/* ---- Tree verification for the 27B-class target (additive: the reference runs this pass as a ggml graph,
 * models/qwen35_27b/src/qwen35_target_graph.cpp:281-804, with the tree logic in models/qwen35_27b/test/test_dflash.cpp).
 * One call evaluates the n_nodes nodes of a draft tree (DFS order, node 0 = root, parents[t] < t, -1 for the root)
 * on top of `past` committed tokens; a node's result is that of the sequential model on its root-to-node path.
 * Layer il is full attention when il % fa_period == fa_period - 1, else DeltaNet.  head_dim must be 256 and the
 * DeltaNet head size 128; hidden and ffn multiples of 256; n_nodes <= 40. */
typedef struct {
    int n_layers, hidden, ffn, vocab;
    int q_heads, kv_heads, head_dim;
    int dn_k_heads, dn_v_heads, dn_dim;
    int rot_dim, fa_period;
    float rope_theta, rms_eps;
} Qwen35TreeDims;

/* Weights of one layer.  Q4_K matrices are row-major arrays of 144-byte super-blocks (256 weights each), rows of the
 * fused matrices concatenated (a GGUF loader concatenates the tensors' bytes: attn_q|attn_k|attn_v, attn_qkv|attn_gate,
 * ffn_gate|ffn_up; tensor names src/gguf_target_loader.cpp:7-39).  Norm and SSM vectors are f32 as in GGUF.  A matrix
 * whose tensors are stored in another type is handed over dequantised to plain bf16 and flagged in dense_mask. */
typedef struct {
    const void* attn_norm;   /* f32 [hidden], applied as a plain multiply */
    const void* post_norm;   /* f32 [hidden] */
    const void* w_in;        /* Q4_K; FA: [2*q_heads*256 + 2*kv_heads*256, hidden], rows [per head q|gate][k][v]; DN: [conv_ch + v_heads*128, hidden], rows [q k v][z] */
    const void* w_ba;        /* DN: bf16 [2*v_heads, hidden], rows [beta ; alpha] */
    const void* w_out;       /* Q4_K [hidden, q_heads*256] or [hidden, v_heads*128] */
    const void* w_gate_up;   /* Q4_K [2*ffn, hidden], rows [gate ; up] */
    const void* w_down;      /* Q4_K [hidden, ffn] */
    const void* q_norm;      /* FA: f32 [256] */
    const void* k_norm;      /* FA: f32 [256] */
    const void* conv_w;      /* DN: f32 [conv_ch][4], tap 3 multiplies the current input */
    const void* ssm_a;       /* DN: f32 [v_heads], -exp(A_log) */
    const void* dt_bias;     /* DN: f32 [v_heads] */
    const void* ssm_norm;    /* DN: f32 [128] */
    unsigned long long dense_mask;   /* bit 0 w_in, 1 w_out, 2 w_gate_up, 3 w_down: that matrix is plain bf16 [rows][cols], not Q4_K */
    const void* reserved[2];
} Qwen35TreeLayer;

typedef struct {
    Qwen35TreeDims dims;
    const Qwen35TreeLayer* layers;   /* HOST array [n_layers] of device pointers */
    const void* token_embd;          /* Q4_K [vocab, hidden] */
    const void* output_norm;         /* f32 [hidden] */
    const void* output_w;            /* Q4_K [vocab, hidden] */
    int n_nodes; int max_nodes;      /* nodes in this tree; node capacity of node_states / node_conv */
    const int* node_tokens;          /* device int32 [n_nodes] */
    const int* parents;              /* device int32 [n_nodes] */
    int past; int max_ctx;           /* committed tokens; cache capacity (past + n_nodes <= max_ctx) */
    void* k_cache; void* v_cache;    /* bf16 [n_fa][kv_heads][max_ctx][256] (or rows of another type, see kv_type); node t is written at slot past + t */
    void* ssm_state;                 /* f32 [n_dn][v_heads][128 value][128 key] */
    void* conv_state;                /* f32 [n_dn][3][conv_ch], row 2 newest */
    void* node_states;               /* f16 [n_dn][max_nodes][v_heads][128][128]: every node's post-state */
    void* node_conv;                 /* f32 [n_dn][max_nodes][conv_ch]: every node's conv input row */
    int* node_argmax;                /* device int32 [n_nodes] out */
    void* logits_out;                /* optional bf16 [n_nodes][vocab] */
    void* dbg_hidden;                /* optional bf16 [n_layers][n_nodes][hidden] */
    int dbg_num_layers;              /* > 0: stop after this many layers (the head still runs) */
    void* scratch; size_t scratch_bytes;   /* caller-owned, >= qwen35_b200_tree_scratch_bytes() */
    const void* dbg_teacher;         /* optional bf16 [n_layers][n_nodes][hidden]: layer l > 0 reads row block l as its input */
    unsigned int dense_mask;         /* bit 0: token_embd is plain bf16 [vocab][hidden]; bit 1: output_w is */
    /* Feature capture for the draft (qwen35_target_graph.cpp:743-787): when target_feat is given, the output of layer
     * capture_layers[k] for node t is written to row (past + t) % feat_cap, columns [k*hidden, (k+1)*hidden) of the
     * ring; tree_commit moves the accepted nodes' rows to positions past, past+1, ... (test_dflash.cpp:1455-1480). */
    void* target_feat;               /* optional bf16 [feat_cap][n_capture * hidden] */
    int feat_cap;                    /* ring capacity in positions */
    int n_capture;                   /* 0..8 captured layers */
    int capture_layers[8];           /* layer indices, ascending (the reference's target: 1, 16, 31, 46, 61) */
    /* 0: k_cache / v_cache rows are bf16 [256].  The reference's cache types (qwen35_target_graph.cpp:110-122):
     * 1: Q8_0, its default: rows of 8 blocks {f16 d, 32 x int8} = 272 bytes, caches uint8 [n_fa][kv_heads][max_ctx][272];
     * 2: Q4_0: rows of 8 blocks {f16 d, 16 bytes of 4-bit codes} = 144 bytes, caches uint8 [..][144];
     * 3: F16 rows [256].
     * A row is converted from its f32 values when written and read as the bf16 operand bf16(value). */
    int kv_type;
} Qwen35TreeVerifyArgs;

size_t qwen35_b200_tree_scratch_bytes(const Qwen35TreeDims* dims, int n_nodes, int max_ctx);
int qwen35_b200_tree_verify(const Qwen35TreeVerifyArgs* args, qwen35_stream_t stream);
/* follow_verified_tree (test_dflash.cpp:396-415) on the device: path[i] = DFS index of the i-th accepted node
 * (path[0] = 0), result[0] = accepted length, result[1] = the next token (arg-max of the last accepted node). */
int qwen35_b200_tree_accept(const int* node_tokens, const int* parents, const int* node_argmax, int n_nodes, int* path, int* result,
                            qwen35_stream_t stream);
/* The commit of test_dflash.cpp:1355-1521, reading path / result from device memory (no host round trip): recurrent
 * state <- persisted f16 state of the last accepted node, conv state <- the last three inputs along the accepted
 * chain, K/V rows of the accepted nodes compacted to slots past, past+1, ...  The caller then adds result[0] to past. */
int qwen35_b200_tree_commit(const Qwen35TreeVerifyArgs* args, const int* path, const int* result, qwen35_stream_t stream);
/* Q4_K super-blocks -> f32 (bit-exact with the published dequantisation (d*sc)*q - dmin*m) and / or bf16. */
int qwen35_b200_dequant_q4k(const void* blocks, size_t n_blocks, void* out_f32, void* out_bf16, qwen35_stream_t stream);

/* Draft side of the speculative loop.  draft_topk: per position, the k largest logits / temperature as log-
 * probabilities (log-sum-exp over the vocabulary) and their token ids, sorted by descending value and ascending id
 * among equals, computed on the GPU (replaces the OpenMP pass extract_draft_topk, test_dflash.cpp:143-207).
 * logits f32 [n_positions][vocab] on the device; outputs [n_positions][k] on the device; 1 <= k <= 16. */
int qwen35_b200_draft_topk(const float* logits, int n_positions, int vocab, int k, float temperature, float* out_log_probs,
                           int* out_token_ids, qwen35_stream_t stream);
/* build_ddtree (test_dflash.cpp:218-390) on the host: best-first tree over prefixes of the per-depth top-k lists
 * (HOST arrays [depth_max][k]), at most `budget` nodes beside the root, optional rank-0 chain first.  Outputs are HOST
 * arrays of 1 + budget entries, node 0 = root (token -1, depth 0, parent -1), parents[i] < i; visibility (optional)
 * is the (1+n)^2 ancestor-or-self matrix.  Returns the number of nodes beside the root, or -1 on bad arguments.  The
 * token / parent arrays are what qwen35_b200_tree_verify takes (after the caller puts the root token in slot 0). */
int qwen35_b200_build_ddtree(const float* top_log_probs, const int* top_token_ids, int depth_max, int k, int budget, int chain_seed,
                             int* token_ids, int* depths, int* parents, unsigned char* visibility);

/* DFlash draft forward: the 5-layer non-causal block-diffusion draft that proposes q_len tokens from the target's captured
 * features (build_draft_graph, models/qwen35_27b/src/qwen3_dflash_graph.cpp:38-166; weights DraftWeights / DraftLayer,
 * src/internal.h).  Stateless like the reference (no KV cache): every call projects the whole feature window.
 *   target_feat = rms_norm(fc . target_hidden_cat) * hidden_norm                       [ctx_len][hidden]
 *   per layer:  Q = wq . norm(h) (per-head RMSNorm, NEOX RoPE at ctx_len + i);  K, V = wk, wv . [target_feat ; norm(h)]
 *               (K per-head RMSNorm, NEOX RoPE at 0 .. ctx_len + q_len - 1);  non-causal attention over all keys, scale
 *               1/sqrt(head_dim);  h += wo . attn;  h += w_down . (silu(w_gate . norm(h)) * (w_up . norm(h)))
 *   hidden_out = rms_norm(h) * out_norm;  optional logits = lm_head . hidden_out (the target's head, bf16 or Q4_K)
 * All matrices are bf16 [out][in] on the device; wkv is the row concatenation [wk ; wv], w_gate_up is [w_gate ; w_up];
 * norm weights are f32 and multiply plainly.  head_dim must be 128, q_len * (n_heads / n_kv_heads) <= 64, hidden and
 * inter multiples of 256.  Every module output is rounded once to bf16 (the reference keeps f32 activations between
 * ggml ops; bf16 storage is this build's convention on every path). */
typedef struct Qwen35DraftDims {
    int hidden, n_layers, n_heads, n_kv_heads, head_dim, inter, n_target_layers, q_len;
    float eps, rope_theta;
} Qwen35DraftDims;
typedef struct Qwen35DraftLayer {
    const void* attn_norm;   /* f32 [hidden] */
    const void* wq;          /* bf16 [n_heads * head_dim][hidden] */
    const void* wkv;         /* bf16 [2 * n_kv_heads * head_dim][hidden]: k rows, then v rows */
    const void* q_norm;      /* f32 [head_dim] */
    const void* k_norm;      /* f32 [head_dim] */
    const void* wo;          /* bf16 [hidden][n_heads * head_dim] */
    const void* ffn_norm;    /* f32 [hidden] */
    const void* w_gate_up;   /* bf16 [2 * inter][hidden]: gate rows, then up rows */
    const void* w_down;      /* bf16 [hidden][inter] */
} Qwen35DraftLayer;
typedef struct Qwen35DraftArgs {
    Qwen35DraftDims dims;
    const Qwen35DraftLayer* layers;      /* HOST array [n_layers] of device pointers */
    const void* fc;                      /* bf16 [hidden][n_target_layers * hidden] */
    const void* hidden_norm;             /* f32 [hidden] */
    const void* out_norm;                /* f32 [hidden] */
    const void* noise_embed;             /* bf16 [q_len][hidden]: the target's embedding of [last token, MASK x (q_len-1)] */
    const void* target_hidden_cat;       /* bf16 [ctx_len][n_target_layers * hidden] */
    int ctx_len;                         /* >= 0 */
    void* hidden_out;                    /* bf16 [q_len][hidden] */
    const void* lm_head;                 /* optional: [vocab][hidden] bf16, or Q4_K super-blocks when lm_head_q4k != 0 */
    int lm_head_q4k;
    int vocab;
    void* logits_out;                    /* bf16 [q_len][vocab] when lm_head is given */
    void* scratch;                       /* device, >= qwen35_b200_draft_scratch_bytes(dims, ctx_len) */
    size_t scratch_bytes;
    qwen35_stream_t stream;
} Qwen35DraftArgs;
size_t qwen35_b200_draft_scratch_bytes(const Qwen35DraftDims* dims, int max_ctx_len);
int qwen35_b200_draft_forward(const Qwen35DraftArgs* args);

/* The prefill and batched-decode entry points keep a host copy of the device pointer tables, keyed by the two
 * table addresses, exactly as the reference keeps its host copy (prefill.cu:1179-1195): after the first call they
 * neither synchronise nor allocate.  A caller that frees its tables and packs new ones may get the same addresses
 * back; it calls this after re-packing so the next call reads the tables again.  No reference counterpart. */
void qwen35_b200_forget_tables(void);

/* BF16 GEMM on tcgen05/TMEM tensor cores: C[M,N] = epi(A[M,K] . B[b_rows,K]^T), f32 accumulate, one
 * rounding to bf16.  Replaces cublas_bf16_gemm (prefill.cu:895-903).  lda/ldc/ldr are row strides in
 * elements; K must be a multiple of 64.  epilogue: 0 = store, 1 = + R (residual, bf16 add),
 * 2 = silu(gate)*up where gate = B rows [0,N) and up = B rows [up_row_offset, up_row_offset+N). */
int qwen35_b200_gemm_bf16(const void* A, int lda, const void* B, int b_rows, void* C, int ldc, const void* R, int ldr,
                          int M, int N, int K, int epilogue, int up_row_offset, qwen35_stream_t stream);

/* The same contraction with Q4_K weights (W = super-blocks [w_rows][K/256][144]), dequantised inside the kernel
 * (the role of ggml_mul_mat on a K-quant tensor, qwen35_target_graph.cpp:262-273, 295-404, 438-661).  M <= 64,
 * K a multiple of 256; rows of W beyond w_rows read as zero. */
int qwen35_b200_gemm_q4k(const void* A, int lda, const void* W, int w_rows, void* C, int ldc, const void* R, int ldr,
                         int M, int N, int K, int epilogue, int up_row_offset, qwen35_stream_t stream);

/* NVFP4 block-scaled GEMM on the tensor cores (tcgen05.mma kind::mxf4nvf4, 16-element blocks, UE4M3 scales, f32 accumulate):
 * C[tokens, n_rows] = alpha * (A_q . W_q^T).  Replaces the reference's cuBLASLt NVFP4 calls: the FP4 LM head
 * (kernel_gb10_nvfp4.cu:277-473, 1894-1997, which quantises the activation to FP4 as well) and the NVFP4 prefill projections
 * (cublaslt_nvfp4_bf16_gemm, prefill.cu:1020-1155).  Both operands are in the layout of launch_quantize_nvfp4_lm_out: packed
 * nibbles [rows, K/2] and scale atoms of 512 bytes (128 rows x 4 scales), atoms of a 128-row block consecutive along K.
 * Weights need n_rows % 128 == 0 and K % 256 == 0.  Activations are packed by qwen35_b200_quantize_act_nvfp4 (bf16 [tokens, K]
 * in; rows are padded to a multiple of 128 with zeros; qwen35_b200_nvfp4_act_bytes gives the two buffer sizes).
 * C is bf16 (one rounding; optional bf16 residual R added after it) or, with out_f32 != 0, f32 without rounding. */
size_t qwen35_b200_nvfp4_act_bytes(int tokens, int K, size_t* scales_bytes);
int qwen35_b200_quantize_act_nvfp4(const void* x, int tokens, int K, void* packed_out, void* scales_out, qwen35_stream_t stream);
int qwen35_b200_gemm_nvfp4(const void* a_packed, const void* a_scales, int tokens, const void* w_packed, const void* w_scales, int n_rows,
                           int K, float alpha, void* C, int ldc, int out_f32, const void* R, int ldr, qwen35_stream_t stream);

/* No counterpart in the reference.  qwen35_b200_decode_steps for callers that must not allocate: an
 * inference server that hands all device memory to its own pool at start-up (a later cudaMalloc inside a
 * library can then fail or fragment the pool), or a latency-critical loop in which the device-wide
 * synchronisation of cudaMalloc/cudaFree would stall other streams.  The megakernel's inter-stage scratch
 * is a fixed array of sizeof(StreamWorkspace) (about 0.6 MB) compiled into the library image; every GPU
 * that loads the library holds one copy until the process exits.  The entry point calls no cudaMalloc,
 * cudaFree or other allocating routine.
 *   - Limit: max_seq_len <= 32768 tokens (what the array is sized for); larger values are rejected with
 *     QWEN35_ERR_BAD_ARG and a message naming the limit.  Inputs, caches and outputs are the caller's.
 *   - The first call on a device looks up the array's device address (cudaGetSymbolAddress with that
 *     device current); make that first call before any stream capture.
 *   - All calls on a device share the one array and it keeps what the previous call wrote.  Stale words
 *     are harmless because every word carries a call-specific epoch; the library clears the array itself
 *     when the 32-bit epoch wraps.  Two calls that overlap on the GPU (different streams) race on the
 *     array: serialise them.  The sticky status word of this array is included in qwen35_b200_status(). */
int qwen35_b200_decode_steps_static(const Qwen35DecodeArgs* args, qwen35_stream_t stream);

/* Synchronises `stream`, then returns the sticky device status word of the current device
 * (QWEN35_OK, or the first error a kernel recorded).  qwen35_b200_clear_status() re-arms the
 * library after an error. */
int qwen35_b200_status(qwen35_stream_t stream);
int qwen35_b200_clear_status(qwen35_stream_t stream);
/* Both read / clear only the status words that exist already: neither creates the library workspace, so a process that
 * uses only qwen35_b200_decode_steps_static never allocates through them.  qwen35_b200_workspace_if_any() returns the
 * workspace of the current device, or NULL while no call has created it (a test hook for exactly that property). */
const void* qwen35_b200_workspace_if_any(void);

/* Debug: synchronise the device and copy one inter-stage vector of the workspace to the host.
 * which: 0 = stage-A output (8224 bf16), 1 = DeltaNet core output (2048 bf16), 2 = hidden after the
 * mixer residual (1024 bf16), 3 = silu(gate)*up (3584 bf16), 4 = layer output (1024 bf16). */
int qwen35_b200_debug_read(int which, void* host_out);

/* Copies the 32 RoPE inverse frequencies the kernels use to a host buffer (for tests). */
int qwen35_b200_rope_inv_freq(float* host_out32);

/* Number of kernels this library has launched in this process (bench bookkeeping). */
long long qwen35_b200_launch_count(void);

const char* qwen35_b200_last_error(void);

#ifdef __cplusplus
}
#endif
#endif /* QWEN35_B200_H */
