// Building blocks of the streaming BF16 decode megakernel (sm_100a):
//   * a per-CTA ring of 16 KB shared-memory slots that a producer warp keeps full with TMA bulk
//     copies (cp.async.bulk + mbarrier complete_tx) of this CTA's weight rows, running ahead of
//     the consumers across stage and layer boundaries;
//   * "flagged words": every value one stage hands to the next travels through L2 as a 64-bit
//     word {payload, epoch}.  A consumer polls the word itself, so one L2 round trip delivers
//     both the data and the proof that it is current -- no grid barrier, no fence on the path.
#pragma once

#include <cuda_fp16.h>
#include <cuda_fp4.h>
#include <cuda_fp8.h>

#include "common.cuh"

namespace q35 {


constexpr int MAX_CTX = 32768;          // longest context the decode scratch is sized for
constexpr int ATT_MAX_CHUNKS = 64;      // split-KV factor of decode attention (chunks per kv head)
constexpr int ATT_CHUNK_MAX = 512;      // longest chunk: MAX_CTX / ATT_MAX_CHUNKS

constexpr int NCONS_WARPS = 16;
constexpr int NCONS = NCONS_WARPS * 32;             // 512 consumer threads
// + one producer warp (weight stream) + one service warp (cache / conv-window updates and their fences, off the consumers' path)
constexpr int STREAM_THREADS = NCONS + 64;
constexpr int SLOT_BYTES = 16384;
constexpr int NSLOTS = 12;

// tiles (one TMA copy each) per stage, whole model
constexpr int TILES_A_DN = DN_PROJ_ROWS / 8;        // 1028 tiles of 8 rows x 1024
constexpr int TILES_A_FA = FA_PROJ_ROWS / 8;        // 640
constexpr int TILES_C = HIDDEN / 4;                 // 256 tiles of 4 rows x 2048
constexpr int UNITS_D = INTER / 8;                  // 448 units = gate tile + up tile (8 rows x 1024 each)
constexpr int TILES_E = HIDDEN / 2;                 // 512 tiles of 2 rows x 3584 (14336 B)
constexpr int TILES_LM = VOCAB / 8;                 // 31040 tiles of 8 rows x 1024

// Library-owned scratch, one per device.  Flagged-word arrays hold two bf16 per word unless noted.
struct StreamWorkspace {
    int err;
    int pad0[63];
    alignas(256) u64 xa[DN_PROJ_ROWS / 2 + 16];     // stage A output: DN [qkv|z|b|a], FA [q,gate|k|v]
    alignas(256) u64 o[FA_Q_SIZE / 2];              // DN: recurrence output; FA: gated attention output
    alignas(256) u64 h1[HIDDEN / 2];                // hidden after the mixer residual
    alignas(256) u64 m[INTER / 2];                  // silu(gate) * up
    alignas(256) u64 h2[HIDDEN / 2];                // layer output
    alignas(256) u64 lm[2][1024];                   // per CTA: {bf16 max bits, epoch}, {arg-max, epoch}
    alignas(256) u64 att_part[ATT_MAX_CHUNKS][FA_Q_HEADS][FA_HEAD_DIM];   // per chunk: f32 partial of P.V, one flagged word per value
    alignas(256) u64 att_stat[FA_Q_HEADS][ATT_MAX_CHUNKS][2];   // per head and chunk: {max, epoch}, {sum exp, epoch}
};

struct DecodeArgs {
    const void* layers;       // device table: LayerWeights (bf16) or LayerWeightsNVFP4 records
    const bf16* embed;
    const bf16* final_norm;
    const bf16* lm_head;      // bf16 [V,1024], or packed E2M1 [V,512] for NVFP4
    const void* lm_scales;    // NVFP4: swizzled E4M3 block scales of the LM head (tensor-core layout)
    bf16* k_cache;
    bf16* v_cache;
    float* dn_states;
    float* conv_bufs;
    StreamWorkspace* ws;
    const int* token_in;      // device pointer to the first input token, or null -> token_imm
    int token_imm;
    const int* forced_ids;    // optional [n_steps]: input token of every step (prefill / teacher forcing)
    int* out_token;           // [1] arg-max of the last step
    int* out_tokens;          // optional [n_steps] arg-max of every step that ran the LM head
    float* logits_out;        // optional [VOCAB] (last step) bf16-rounded logits widened to f32
    bf16* hidden_out;         // optional [HIDDEN]: last layer's output of the last step
    bf16* dbg_hidden;         // optional [NUM_LAYERS][HIDDEN]: every layer's output of the last step
    const bf16* dbg_teacher;  // optional [NUM_LAYERS][HIDDEN]: input of layer l>0 is row l instead of the previous layer's output
    unsigned long long* dbg_time;  // optional [25][12]: %globaltimer stamps of CTA dbg_time_cta, last step
    int dbg_time_cta;
    int position;             // tokens already cached
    int max_seq_len;
    int n_steps;
    int lm_last_only;         // 1: LM head only after the last step (prefill)
    int dbg_num_layers;       // 0 = all; otherwise stop after this many layers
    int tma_period;           // minimum SM clocks between two weight-tile copies of one CTA (paces the HBM stream)
    unsigned epoch_base;      // epochs used by this launch: epoch_base + 32*step + {1..24 layer, 25 LM}
};

// ---- flagged words --------------------------------------------------------------------------------
__device__ __forceinline__ u64 ld_word(const u64* p) {
    u64 v;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_word(u64* p, uint32_t payload, uint32_t epoch) {
    const u64 v = ((u64)epoch << 32) | (u64)payload;
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
    const __nv_bfloat162 t = __halves2bfloat162(f2bf(lo), f2bf(hi));
    return *reinterpret_cast<const uint32_t*>(&t);
}

constexpr unsigned POLL_LIMIT = 3u * 1000u * 1000u;
#ifndef POLL_BACKOFF_NS
#define POLL_BACKOFF_NS 0
#endif

// Shared abort protocol: the first wait that runs out records an error and raises `*s_abort`;
// after that no wait blocks, so every thread runs to the end of the kernel and exits normally.
struct Abort {
    volatile int* s_abort;
    int* g_err;
    __device__ __forceinline__ bool on() const { return *s_abort != 0; }
    __device__ __forceinline__ void raise(int code) const {
        *s_abort = 1;
        atomicCAS(g_err, 0, code);
    }
};

__device__ __forceinline__ uint32_t poll_word(const u64* p, uint32_t epoch, const Abort& ab) {
    u64 v = ld_word(p);
    if ((uint32_t)(v >> 32) == epoch) return (uint32_t)v;
    unsigned it = 0;
    while (!ab.on()) {
        if (POLL_BACKOFF_NS) __nanosleep(POLL_BACKOFF_NS);
        v = ld_word(p);
        if ((uint32_t)(v >> 32) == epoch) break;
        if (++it > POLL_LIMIT || ((it & 4095u) == 0 && ld_volatile(ab.g_err) != 0)) { ab.raise(ERR_BARRIER_TIMEOUT); break; }
    }
    return (uint32_t)v;
}

// N words `stride` apart (only the first `n` are live).  Every round re-issues the loads of all
// words that are still stale together, so a late producer costs one L2 round trip, not N.
template <int N>
__device__ __forceinline__ void poll_n(const u64* p, int stride, int n, uint32_t epoch, const Abort& ab, uint32_t (&o)[N]) {
    u64 v[N];
    unsigned pending = 0;
#pragma unroll
    for (int i = 0; i < N; ++i) if (i < n) v[i] = ld_word(p + i * stride);
#pragma unroll
    for (int i = 0; i < N; ++i) if (i < n && (uint32_t)(v[i] >> 32) != epoch) pending |= 1u << i;
    unsigned it = 0;
    while (pending && !ab.on()) {
        if (POLL_BACKOFF_NS) __nanosleep(POLL_BACKOFF_NS);
#pragma unroll
        for (int i = 0; i < N; ++i) if (pending & (1u << i)) v[i] = ld_word(p + i * stride);
#pragma unroll
        for (int i = 0; i < N; ++i) if ((pending & (1u << i)) && (uint32_t)(v[i] >> 32) == epoch) pending &= ~(1u << i);
        if (++it > POLL_LIMIT || ((it & 4095u) == 0 && ld_volatile(ab.g_err) != 0)) { ab.raise(ERR_BARRIER_TIMEOUT); break; }
    }
#pragma unroll
    for (int i = 0; i < N; ++i) o[i] = (uint32_t)v[i];
}

// N units of two adjacent words, the units `stride` words apart (only the first `n` units are live): o[2 i], o[2 i + 1].
template <int N>
__device__ __forceinline__ void poll_pairs(const u64* p, int stride, int n, uint32_t epoch, const Abort& ab, uint32_t (&o)[2 * N]) {
    u64 v[2 * N];
    unsigned pending = 0;
#pragma unroll
    for (int i = 0; i < 2 * N; ++i) if ((i >> 1) < n) v[i] = ld_word(p + (i >> 1) * stride + (i & 1));
#pragma unroll
    for (int i = 0; i < 2 * N; ++i) if ((i >> 1) < n && (uint32_t)(v[i] >> 32) != epoch) pending |= 1u << i;
    unsigned it = 0;
    while (pending && !ab.on()) {
#pragma unroll
        for (int i = 0; i < 2 * N; ++i) if (pending & (1u << i)) v[i] = ld_word(p + (i >> 1) * stride + (i & 1));
#pragma unroll
        for (int i = 0; i < 2 * N; ++i) if ((pending & (1u << i)) && (uint32_t)(v[i] >> 32) == epoch) pending &= ~(1u << i);
        if (++it > POLL_LIMIT || ((it & 4095u) == 0 && ld_volatile(ab.g_err) != 0)) { ab.raise(ERR_BARRIER_TIMEOUT); break; }
    }
#pragma unroll
    for (int i = 0; i < 2 * N; ++i) o[i] = ((i >> 1) < n) ? (uint32_t)v[i] : 0u;
}

__device__ __forceinline__ void mbar_wait(uint32_t bar, uint32_t parity, const Abort& ab) {
    unsigned it = 0;
    while (!mbar_try_wait(bar, parity)) {
        if (ab.on()) return;
        if (++it > POLL_LIMIT) { ab.raise(ERR_BARRIER_TIMEOUT); return; }
    }
}

// consumer-only barrier (the producer warp never joins it)
__device__ __forceinline__ void cons_sync() { asm volatile("bar.sync 1, %0;" ::"n"(NCONS) : "memory"); }

__device__ __forceinline__ float cons_block_sum(float v, float* scratch) {
    v = warp_sum(v);
    cons_sync();
    if ((threadIdx.x & 31) == 0) scratch[threadIdx.x >> 5] = v;
    cons_sync();
    float t = 0.f;
#pragma unroll
    for (int i = 0; i < NCONS_WARPS; ++i) t += scratch[i];
    return t;
}

// Ring bookkeeping shared by the producer and the consumers: tiles are numbered in issue order.
struct Ring {
    uint32_t slots;      // shared address of slot 0
    uint32_t full;       // shared address of full[0]
    uint32_t empty;      // shared address of empty[0]
    unsigned t;          // running tile counter
    __device__ __forceinline__ uint32_t slot_addr(unsigned tile) const { return slots + (tile % NSLOTS) * SLOT_BYTES; }
    __device__ __forceinline__ uint32_t full_bar(unsigned tile) const { return full + (tile % NSLOTS) * 8; }
    __device__ __forceinline__ uint32_t empty_bar(unsigned tile) const { return empty + (tile % NSLOTS) * 8; }
    __device__ __forceinline__ uint32_t phase(unsigned tile) const { return (tile / NSLOTS) & 1u; }
};

// dot of 8 bf16 weights (one 16-byte chunk) with 8 f32 activations
__device__ __forceinline__ float dot8(const uint4 q, const float* x, float a) {
    a = fmaf(bf_lo(q.x), x[0], a); a = fmaf(bf_hi(q.x), x[1], a);
    a = fmaf(bf_lo(q.y), x[2], a); a = fmaf(bf_hi(q.y), x[3], a);
    a = fmaf(bf_lo(q.z), x[4], a); a = fmaf(bf_hi(q.z), x[5], a);
    a = fmaf(bf_lo(q.w), x[6], a); a = fmaf(bf_hi(q.w), x[7], a);
    return a;
}
__device__ __forceinline__ float dot8p(const uint4 q, const uint4 y, float a) {
    a = fmaf(bf_lo(q.x), bf_lo(y.x), a); a = fmaf(bf_hi(q.x), bf_hi(y.x), a);
    a = fmaf(bf_lo(q.y), bf_lo(y.y), a); a = fmaf(bf_hi(q.y), bf_hi(y.y), a);
    a = fmaf(bf_lo(q.z), bf_lo(y.z), a); a = fmaf(bf_hi(q.z), bf_hi(y.z), a);
    a = fmaf(bf_lo(q.w), bf_lo(y.w), a); a = fmaf(bf_hi(q.w), bf_hi(y.w), a);
    return a;
}
// d = a_lo * b_lo + a_hi * b_hi + d for two packed bf16 pairs, f32 accumulate: the mixed-precision FMA of sm_100
// (fma.rn.f32.bf16) takes its bf16 operands as they are, so no conversion instruction precedes it.  A product of two
// bf16 values is exact in f32, hence each step rounds once, exactly like fmaf on the widened values.
__device__ __forceinline__ float fma2_bf16(uint32_t a, uint32_t b, float d) {
    asm("{\n\t.reg .b16 al, ah, bl, bh;\n\t"
        "mov.b32 {al, ah}, %1;\n\t"
        "mov.b32 {bl, bh}, %2;\n\t"
        "fma.rn.f32.bf16 %0, al, bl, %0;\n\t"
        "fma.rn.f32.bf16 %0, ah, bh, %0;\n\t}"
        : "+f"(d) : "r"(a), "r"(b));
    return d;
}
// 8 bf16 weights (one 16-byte chunk) times 8 bf16 activations (packed the same way)
__device__ __forceinline__ float dot8m(const uint4 w, const uint4 y, float a) {
    a = fma2_bf16(w.x, y.x, a);
    a = fma2_bf16(w.y, y.y, a);
    a = fma2_bf16(w.z, y.z, a);
    return fma2_bf16(w.w, y.w, a);
}
// Sums two per-lane values over the warp with five shuffles instead of ten: after the first exchange lanes 0-15 carry
// `a`, lanes 16-31 carry `b`; on return every lane below 16 holds the total of a, every lane from 16 up the total of b.
__device__ __forceinline__ float warp_sum2(float a, float b) {
    const bool hi = (threadIdx.x & 16) != 0;
    float keep = hi ? b : a;
    const float send = hi ? a : b;
    keep += __shfl_xor_sync(0xffffffffu, send, 16);
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) keep += __shfl_xor_sync(0xffffffffu, keep, o);
    return keep;
}

__device__ __forceinline__ void unpack8(const uint4 v, float* x) {
    x[0] = bf_lo(v.x); x[1] = bf_hi(v.x); x[2] = bf_lo(v.y); x[3] = bf_hi(v.y);
    x[4] = bf_lo(v.z); x[5] = bf_hi(v.z); x[6] = bf_lo(v.w); x[7] = bf_hi(v.w);
}
__device__ __forceinline__ uint4 lds128(uint32_t addr) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
    return v;
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
