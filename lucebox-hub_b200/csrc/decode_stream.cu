// Streaming BF16 decode megakernel for the Qwen3.5-0.8B hybrid network (sm_100a).
//
// Replaces models/qwen35_0p8b/kernel.cu of the reference (decode_kernel :820-904, the layer
// bodies :409-741, lm_head_kernel :747-814, launch_decode :910-1020).  One persistent
// cooperative launch (one CTA per SM) runs all 24 layers and the LM-head arg-max for one or
// many tokens.  Per CTA:
//   * warp 16 is a TMA producer.  It walks this CTA's static list of weight tiles (16 KB,
//     contiguous rows of one matrix) for every stage of every layer and keeps a 12-slot
//     shared-memory ring full with cp.async.bulk copies, never waiting for activations, so HBM
//     keeps streaming while the consumers wait for the previous stage;
//   * warps 0-15 are consumers.  A stage waits for its input vector by polling flagged 64-bit
//     words {two bf16, epoch} that the previous stage's CTAs wrote straight to L2, computes its
//     rows from shared memory, and publishes its outputs the same way.  There is no grid
//     barrier anywhere on the path.
// Stages per layer: A input norm + fused projection; B DeltaNet recurrence (all CTAs, one warp
// per pair of value rows) or attention (B1 scores, B2 P.V partials, B3 merge+gate on a few
// CTAs); C gated norm / copy + output projection + residual; D post norm + gate/up with
// SiLU*up; E down projection + residual.  Numerics are those of a bf16 HuggingFace model.
#include "decode_stream.cuh"

#include <cooperative_groups.h>

namespace q35 {

// 1 / theta^(2i/64), i = 0..31, theta = 1e7 (the reference evaluates powf per call, kernel.cu:483-490);
// filled by the host from a double-precision pow so that it equals torch's f32 table bit for bit.
__constant__ float c_rope_inv_freq[FA_ROT / 2];

// Layer pointers in one order for both weight formats.  *S slots are the block scales of the NVFP4 format
// (null for bf16).  A0..A3 are the stage-A matrices: DeltaNet qkv, z, b, a; attention q, k, v.
enum WSlot { W_IN_NORM = 0, W_POST_NORM, W_A0, W_A0S, W_A1, W_A1S, W_A2, W_A2S, W_A3, W_CONV, W_ALOG, W_DTBIAS, W_GNORM,
             W_QNORM, W_KNORM, W_OUT, W_OUTS, W_GATE, W_GATES, W_UP, W_UPS, W_DOWN, W_DOWNS, W_NSLOTS };
struct LayerW {
    int type;
    int pad;
    const void* p[W_NSLOTS];
};

// bf16 table: struct LayerWeights (kernel.cu:77-115); NVFP4 table: struct LayerWeightsNVFP4
// {int type; int group_size; int pad[2]; void* ptrs[24]} with the slot order of model.py:248-284.
template <bool FP4>
__device__ __forceinline__ void load_layer(const void* table, int layer, LayerW& out) {
    constexpr int REC = FP4 ? 208 : 128;
    const char* rec = (const char*)table + (size_t)layer * REC;
    const int type = *reinterpret_cast<const int*>(rec);
    const void* const* r = reinterpret_cast<const void* const*>(rec + 16);
    out.type = type;
    for (int i = 0; i < W_NSLOTS; ++i) out.p[i] = nullptr;
    if (!FP4) {
        if (type == 0) {
            out.p[W_IN_NORM] = r[0]; out.p[W_A0] = r[1]; out.p[W_A1] = r[2]; out.p[W_A2] = r[3]; out.p[W_A3] = r[4];
            out.p[W_CONV] = r[5]; out.p[W_ALOG] = r[6]; out.p[W_DTBIAS] = r[7]; out.p[W_GNORM] = r[8]; out.p[W_OUT] = r[9];
            out.p[W_POST_NORM] = r[10]; out.p[W_GATE] = r[11]; out.p[W_UP] = r[12]; out.p[W_DOWN] = r[13];
        } else {
            out.p[W_IN_NORM] = r[0]; out.p[W_A0] = r[1]; out.p[W_A1] = r[2]; out.p[W_A2] = r[3]; out.p[W_QNORM] = r[4];
            out.p[W_KNORM] = r[5]; out.p[W_OUT] = r[6]; out.p[W_POST_NORM] = r[7]; out.p[W_GATE] = r[8]; out.p[W_UP] = r[9];
            out.p[W_DOWN] = r[10];
        }
    } else {
        if (type == 0) {
            out.p[W_IN_NORM] = r[0]; out.p[W_A0] = r[1]; out.p[W_A0S] = r[2]; out.p[W_A1] = r[3]; out.p[W_A1S] = r[4];
            out.p[W_A2] = r[5]; out.p[W_A3] = r[6]; out.p[W_CONV] = r[7]; out.p[W_ALOG] = r[8]; out.p[W_DTBIAS] = r[9];
            out.p[W_GNORM] = r[10]; out.p[W_OUT] = r[11]; out.p[W_OUTS] = r[12]; out.p[W_POST_NORM] = r[13];
            out.p[W_GATE] = r[14]; out.p[W_GATES] = r[15]; out.p[W_UP] = r[16]; out.p[W_UPS] = r[17]; out.p[W_DOWN] = r[18]; out.p[W_DOWNS] = r[19];
        } else {
            out.p[W_IN_NORM] = r[0]; out.p[W_A0] = r[1]; out.p[W_A0S] = r[2]; out.p[W_A1] = r[3]; out.p[W_A1S] = r[4];
            out.p[W_A2] = r[5]; out.p[W_A2S] = r[6]; out.p[W_QNORM] = r[7]; out.p[W_KNORM] = r[8]; out.p[W_OUT] = r[9]; out.p[W_OUTS] = r[10];
            out.p[W_POST_NORM] = r[11]; out.p[W_GATE] = r[12]; out.p[W_GATES] = r[13]; out.p[W_UP] = r[14]; out.p[W_UPS] = r[15];
            out.p[W_DOWN] = r[16]; out.p[W_DOWNS] = r[17];
        }
    }
}

// Work split of one CTA over the stages: contiguous ranges [begin, end) of tiles / units / row pairs.  The bounds need a
// 64-bit multiply and divide each, so they are computed once per launch and kept in shared memory.
enum PartIdx { PT_A_DN0, PT_A_DN1, PT_A_FA0, PT_A_FA1, PT_C0, PT_C1, PT_D0, PT_D1, PT_E0, PT_E1, PT_PAIR0, PT_PAIR1, PT_CS0, PT_CS1,
               PT_LM0, PT_LM1, PT_LMB0, PT_LMB1, PT_COUNT };

struct Smem {
    // ring first: 16-byte aligned slots
    unsigned char ring[NSLOTS * SLOT_BYTES];
    unsigned long long full[NSLOTS];
    unsigned long long empty[NSLOTS];
    unsigned long long side_go;                  // consumers -> service warp, once per layer: the layer's side work may start
    unsigned long long side_done;                // service warp -> consumers: it is done and fenced
    LayerW layers[NUM_LAYERS];
    __align__(16) bf16 x[INTER];                 // GEMV input of the current stage
    __align__(16) bf16 h[HIDDEN];                // raw layer input (residual of stage C)
    __align__(16) bf16 h1[HIDDEN];               // raw mixer output (residual of stage E)
    float part[512];                             // cross-warp partial sums; attention chunk statistics
    uint32_t stage[64];                          // packed outputs of a GEMV stage, published by one coalesced store
    uint32_t stage_b[NCONS_WARPS];               // DeltaNet recurrence outputs
    float red[NCONS_WARPS];
    __align__(16) float qk[2][2][DN_K];          // DeltaNet: normalised q and k of the (at most two) heads this CTA works on
    float hd[2][2];                              // their beta and decay
    int pt[PT_COUNT];                            // this CTA's share of every stage, computed once (see PartIdx)
    int lm_row0[256];                            // first vocabulary row of every CTA's LM-head share (arg-max merge)
    __align__(16) float q[FA_GQA][FA_HEAD_DIM];
    __align__(16) float kcur[FA_HEAD_DIM];
    __align__(16) uint32_t vcur[FA_HEAD_DIM / 2];  // the new value row (packed bf16) of the CTA whose chunk holds the current position
    __align__(16) float p[FA_GQA][ATT_CHUNK_MAX]; // scores, then probabilities, of this CTA's chunk; then the merge's group sums
    float ml[FA_GQA][2];
    int abort_flag;
    int tok;
};

__device__ __forceinline__ unsigned long long gtime() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}
#define Q35_STAMP_ALL(k)                                                                               \
    do {                                                                                               \
        if (a.dbg_time) { cons_sync(); Q35_STAMP(k); }                                                  \
    } while (0)
#define Q35_STAMP(k)                                                                                   \
    do {                                                                                               \
        if (a.dbg_time && last_step && tid == 0)                                                       \
            a.dbg_time[((size_t)b * 25 + stamp_row) * 12 + (k)] = (a.dbg_time_cta == -2) ? (unsigned long long)clock64() : gtime(); \
    } while (0)

__device__ __forceinline__ unsigned epoch_of(const DecodeArgs& a, int step, int slot) {
    return a.epoch_base + 32u * (unsigned)step + (unsigned)slot + 1u;   // slot: 0..23 layer, 24 LM
}

// ------------------------------------------------------------------------------------------------
// producer: issue every weight tile of this CTA in consumption order
// ------------------------------------------------------------------------------------------------
// NVFP4 tile geometry (decode-body layout, group 32: 0.5 byte per weight + one fp16 scale per 32 weights).
// Packed nibbles sit at the start of the slot, the fp16 scales of the same rows at FP4_SCALE_OFF.
constexpr uint32_t FP4_SCALE_OFF = 8192;
constexpr int FP4_LM_BLOCKS = VOCAB / 128;          // LM head (tensor-core layout): 1940 blocks of 128 rows

template <bool FP4>
__device__ __forceinline__ void produce(const DecodeArgs& a, Smem& s, Ring ring, const Abort& ab) {
    const u64 pol = l2_policy_evict_first();
    long long next_t = clock64();
    const long long period = a.tma_period;
    // one tile = one slot: `bytes` from src at the slot start and, for NVFP4, `sbytes` of scales at FP4_SCALE_OFF
    auto issue = [&](const void* src, uint32_t bytes, const void* ssrc, uint32_t sbytes) {
        if (ab.on()) return;                       // after an abort nothing new is put in flight
        const unsigned t = ring.t;
        mbar_wait(ring.empty_bar(t), ring.phase(t) ^ 1u, ab);
        if (ab.on()) return;
        long long now = clock64();
        while (now < next_t) now = clock64();
        next_t = now + period;
        ring.t = t + 1;
        mbar_arrive_expect_tx(ring.full_bar(t), bytes + sbytes);
        tma_load_1d(ring.slot_addr(t), src, bytes, ring.full_bar(t), pol);
        if (sbytes) tma_load_1d(ring.slot_addr(t) + FP4_SCALE_OFF, ssrc, sbytes, ring.full_bar(t), pol);
    };
    // rows [row, row + nrows) of a [*, K] matrix
    auto issue_rows = [&](const void* w, const void* sc, int row, int nrows, int K) {
        if (FP4 && sc) issue((const char*)w + (size_t)row * (K / 2), (uint32_t)(nrows * (K / 2)), (const char*)sc + (size_t)row * (K / 16), (uint32_t)(nrows * (K / 16)));
        else issue((const char*)w + (size_t)row * K * 2, (uint32_t)(nrows * K * 2), nullptr, 0);
    };
    const int n_layers = a.dbg_num_layers > 0 ? a.dbg_num_layers : NUM_LAYERS;
    for (int step = 0; step < a.n_steps; ++step) {
        for (int layer = 0; layer < n_layers; ++layer) {
            const LayerW& L = s.layers[layer];
            if (L.type == 0) {
                for (int u = s.pt[PT_A_DN0]; u < s.pt[PT_A_DN1]; ++u) {
                    const int v = u * 8;
                    if (v < DN_CONV_CH) issue_rows(L.p[W_A0], L.p[W_A0S], v, 8, HIDDEN);
                    else if (v < DN_CONV_CH + DN_V_SIZE) issue_rows(L.p[W_A1], L.p[W_A1S], v - DN_CONV_CH, 8, HIDDEN);
                    else if (v < DN_CONV_CH + DN_V_SIZE + DN_HEADS) issue_rows(L.p[W_A2], nullptr, v - DN_CONV_CH - DN_V_SIZE, 8, HIDDEN);
                    else issue_rows(L.p[W_A3], nullptr, v - DN_CONV_CH - DN_V_SIZE - DN_HEADS, 8, HIDDEN);
                }
            } else {
                for (int u = s.pt[PT_A_FA0]; u < s.pt[PT_A_FA1]; ++u) {
                    const int v = u * 8;
                    if (v < FA_QPROJ) issue_rows(L.p[W_A0], L.p[W_A0S], v, 8, HIDDEN);
                    else if (v < FA_QPROJ + FA_KV_SIZE) issue_rows(L.p[W_A1], L.p[W_A1S], v - FA_QPROJ, 8, HIDDEN);
                    else issue_rows(L.p[W_A2], L.p[W_A2S], v - FA_QPROJ - FA_KV_SIZE, 8, HIDDEN);
                }
            }
            for (int u = s.pt[PT_C0]; u < s.pt[PT_C1]; ++u) issue_rows(L.p[W_OUT], L.p[W_OUTS], u * 4, 4, 2048);
            for (int u = s.pt[PT_D0]; u < s.pt[PT_D1]; ++u) {
                issue_rows(L.p[W_GATE], L.p[W_GATES], u * 8, 8, HIDDEN);
                issue_rows(L.p[W_UP], L.p[W_UPS], u * 8, 8, HIDDEN);
            }
            for (int u = s.pt[PT_E0]; u < s.pt[PT_E1]; ++u) issue_rows(L.p[W_DOWN], L.p[W_DOWNS], u * 2, 2, INTER);
        }
        if (!a.lm_last_only || step == a.n_steps - 1) {
            if (!FP4) {
                for (int u = s.pt[PT_LM0]; u < s.pt[PT_LM1]; ++u)
                    issue((const char*)a.lm_head + (size_t)u * SLOT_BYTES, SLOT_BYTES, nullptr, 0);
            } else {
                // per 128-row block: its 8 KB of swizzled E4M3 scales, then four 32-row tiles of packed nibbles
                for (int blk = s.pt[PT_LMB0]; blk < s.pt[PT_LMB1]; ++blk) {
                    issue((const char*)a.lm_scales + (size_t)blk * 8192, 8192, nullptr, 0);
                    for (int q = 0; q < 4; ++q) issue((const char*)a.lm_head + ((size_t)blk * 128 + q * 32) * 512, 16384, nullptr, 0);
                }
            }
        }
    }
    // drain: every copy this CTA issued must have landed before the CTA may exit
    const unsigned issued = ring.t;
    const unsigned first = issued > NSLOTS ? issued - NSLOTS : 0;
    for (unsigned t = first; t < issued; ++t) {
        unsigned it = 0;
        while (!mbar_try_wait(ring.full_bar(t), ring.phase(t))) {
            if (++it > POLL_LIMIT) { ab.raise(ERR_BARRIER_TIMEOUT); break; }
        }
    }
}

// ------------------------------------------------------------------------------------------------
// consumer helpers
// ------------------------------------------------------------------------------------------------
// K = 1024 rows, 8 per tile: four tiles in flight per CTA, warp w takes tile w/4, rows 2(w%4), +1.
// xq: this lane's activations, packed bf16, chunk j = elements [(32 j + lane) 8, +8) -- the same split as the 16-byte
// chunks of a weight row, so a chunk of weights meets its chunk of activations in one dot8m.
// NMAT = 2 pairs a gate tile with an up tile.  epi(row, sums[NMAT]) runs on lane 0 for the first row of the pair and on
// lane 16 for the second.
template <int NMAT, typename Epi>
__device__ __forceinline__ void consume_k1024(Ring& ring, int n_units, const uint4 (&xq)[4], const Abort& ab, Epi epi) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const unsigned t0 = ring.t;
    for (int g = 0; g < n_units; g += 4) {
        const int ui = g + (warp >> 2);
        if (ui < n_units) {
            float acc[NMAT];
#pragma unroll
            for (int m = 0; m < NMAT; ++m) {
                const unsigned tile = t0 + (unsigned)(ui * NMAT + m);
                mbar_wait(ring.full_bar(tile), ring.phase(tile), ab);
                const uint32_t base = ring.slot_addr(tile) + (uint32_t)(2 * (warp & 3)) * 2048u + (uint32_t)lane * 16u;
                uint4 w0[4], w1[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) { w0[j] = lds128(base + j * 512); w1[j] = lds128(base + 2048 + j * 512); }
                // four independent accumulation chains per warp
                float a0 = dot8m(w0[0], xq[0], 0.f), a1 = dot8m(w0[1], xq[1], 0.f);
                float b0 = dot8m(w1[0], xq[0], 0.f), b1 = dot8m(w1[1], xq[1], 0.f);
                a0 = dot8m(w0[2], xq[2], a0); a1 = dot8m(w0[3], xq[3], a1);
                b0 = dot8m(w1[2], xq[2], b0); b1 = dot8m(w1[3], xq[3], b1);
                acc[m] = warp_sum2(a0 + a1, b0 + b1);
                if (lane == 0) mbar_arrive(ring.empty_bar(tile), 4);
            }
            if ((lane & 15) == 0) epi(ui * 8 + 2 * (warp & 3) + (lane >> 4), acc);
        }
    }
    ring.t = t0 + (unsigned)(n_units * NMAT);
}

// ---- NVFP4 (E2M1 + block scale) dequantisation in registers ----
__device__ __forceinline__ float2 fp4x2_to_float2(uint32_t byte) {
    const __half2_raw h = __nv_cvt_fp4x2_to_halfraw2((__nv_fp4x2_storage_t)byte, __NV_E2M1);   // low nibble -> .x
    return __half22float2(*reinterpret_cast<const __half2*>(&h));
}
// 32 E2M1 weights (16 bytes) times 32 activations, f32 accumulate; the block scale is applied by the caller
__device__ __forceinline__ float dot32_fp4(const uint4 p, const float* x) {
    const uint32_t w[4] = {p.x, p.y, p.z, p.w};
    float a0 = 0.f, a1 = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int bb = 0; bb < 4; ++bb) {
            const float2 f = fp4x2_to_float2((w[i] >> (8 * bb)) & 0xffu);
            a0 = fmaf(f.x, x[i * 8 + bb * 2], a0);
            a1 = fmaf(f.y, x[i * 8 + bb * 2 + 1], a1);
        }
    return a0 + a1;
}
// the two halves (16 weights each) separately: tensor-core layout has one scale per 16 weights
__device__ __forceinline__ float2 dot16x2_fp4(const uint4 p, const float* x) {
    const uint32_t w[4] = {p.x, p.y, p.z, p.w};
    float a[2] = {0.f, 0.f};
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int bb = 0; bb < 4; ++bb) {
            const float2 f = fp4x2_to_float2((w[i] >> (8 * bb)) & 0xffu);
            a[i >> 1] = fmaf(f.x, x[i * 8 + bb * 2], a[i >> 1]);
            a[i >> 1] = fmaf(f.y, x[i * 8 + bb * 2 + 1], a[i >> 1]);
        }
    return make_float2(a[0], a[1]);
}
__device__ __forceinline__ float lds_half(uint32_t addr) {
    unsigned short v;
    asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(addr));
    return __half2float(__ushort_as_half(v));
}
__device__ __forceinline__ float2 lds_e4m3x2(uint32_t addr) {
    unsigned short v;
    asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(addr));
    const __half2_raw h = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)v, __NV_E4M3);
    return __half22float2(*reinterpret_cast<const __half2*>(&h));
}
// 32 consecutive activations starting at element e0 (a multiple of 32)
__device__ __forceinline__ void load_x32(const bf16* xs, int e0, float* x) {
#pragma unroll
    for (int j = 0; j < 4; ++j) unpack8(*reinterpret_cast<const uint4*>(xs + e0 + 8 * j), x + 8 * j);
}

// NVFP4 version of consume_k1024: a row is 512 bytes of nibbles, lane l owns elements [32 l, 32 l + 32), which
// is exactly one scale group, so the scale is applied once per (row, lane) after the dot product.
template <int NMAT, typename Epi>
__device__ __forceinline__ void consume_k1024_fp4(Ring& ring, int n_units, const uint4 (&xc)[4], const Abort& ab, Epi epi) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float x[32];
#pragma unroll
    for (int j = 0; j < 4; ++j) unpack8(xc[j], x + 8 * j);
    const unsigned t0 = ring.t;
    for (int g = 0; g < n_units; g += 4) {
        const int ui = g + (warp >> 2);
        if (ui < n_units) {
            float acc[NMAT];
#pragma unroll
            for (int m = 0; m < NMAT; ++m) {
                const unsigned tile = t0 + (unsigned)(ui * NMAT + m);
                mbar_wait(ring.full_bar(tile), ring.phase(tile), ab);
                const uint32_t r0 = (uint32_t)(2 * (warp & 3));
                const uint32_t base = ring.slot_addr(tile) + r0 * 512u + (uint32_t)lane * 16u;
                const uint32_t sbase = ring.slot_addr(tile) + FP4_SCALE_OFF + r0 * 64u + (uint32_t)lane * 2u;
                const uint4 p0 = lds128(base), p1 = lds128(base + 512);
                const float s0 = lds_half(sbase), s1 = lds_half(sbase + 64);
                acc[m] = warp_sum2(dot32_fp4(p0, x) * s0, dot32_fp4(p1, x) * s1);
                if (lane == 0) mbar_arrive(ring.empty_bar(tile), 4);
            }
            if ((lane & 15) == 0) epi(ui * 8 + 2 * (warp & 3) + (lane >> 4), acc);
        }
    }
    ring.t = t0 + (unsigned)(n_units * NMAT);
}

__device__ __forceinline__ void poll2(const u64* p0, const u64* p1, uint32_t epoch, const Abort& ab, uint32_t& o0, uint32_t& o1) {
    uint32_t o[2];
    poll_n<2>(p0, (int)(p1 - p0), 2, epoch, ab, o);
    o0 = o[0]; o1 = o[1];
}
__device__ __forceinline__ void poll4(const u64* p, int stride, uint32_t epoch, const Abort& ab, uint32_t (&o)[4]) {
    poll_n<4>(p, stride, 4, epoch, ab, o);
}

// N flagged words at arbitrary addresses, all loads of a round in flight together.
template <int N>
__device__ __forceinline__ void poll_ptrs(const u64* const (&p)[N], uint32_t epoch, const Abort& ab, uint32_t (&o)[N]) {
    u64 v[N];
    unsigned pending = 0;
#pragma unroll
    for (int i = 0; i < N; ++i) v[i] = ld_word(p[i]);
#pragma unroll
    for (int i = 0; i < N; ++i) if ((uint32_t)(v[i] >> 32) != epoch) pending |= 1u << i;
    unsigned it = 0;
    while (pending && !ab.on()) {
#pragma unroll
        for (int i = 0; i < N; ++i) if (pending & (1u << i)) v[i] = ld_word(p[i]);
#pragma unroll
        for (int i = 0; i < N; ++i) if ((pending & (1u << i)) && (uint32_t)(v[i] >> 32) == epoch) pending &= ~(1u << i);
        if (++it > POLL_LIMIT || ((it & 4095u) == 0 && ld_volatile(ab.g_err) != 0)) { ab.raise(ERR_BARRIER_TIMEOUT); break; }
    }
#pragma unroll
    for (int i = 0; i < N; ++i) o[i] = (uint32_t)v[i];
}

// Hidden-state hand-off: every consumer thread fetches one flagged word of a [1024] bf16 vector and parks the payload in
// shared memory; the caller's cons_sync() hands them to everybody.  (Fewer polling warps with more words each were
// measured slower: 4 warps -7 %, 2 warps -8 % on tg128.)
__device__ __forceinline__ void fetch_vec1024(const u64* src, uint32_t epoch, bf16* dst, const Abort& ab) {
    const int t = threadIdx.x;
    reinterpret_cast<uint32_t*>(dst)[t] = poll_word(src + t, epoch, ab);
}

// Which 16-byte chunks of a [1024] bf16 vector a lane holds.  Interleaved (bf16 weights): chunk j = elements [(32 j + lane) 8, +8),
// the split of a weight row's 16-byte chunks over the lanes.  Contiguous (NVFP4 weights): elements [32 lane + 8 j, +8), one
// 32-element scale group per lane.
template <bool CONTIG>
__device__ __forceinline__ int lane_chunk(int j) { return CONTIG ? (int)(threadIdx.x & 31) * 4 + j : j * 32 + (int)(threadIdx.x & 31); }

template <bool CONTIG>
__device__ __forceinline__ void load_lane_chunks(const bf16* w, uint4 (&out)[4]) {
#pragma unroll
    for (int j = 0; j < 4; ++j) out[j] = __ldg(reinterpret_cast<const uint4*>(w) + lane_chunk<CONTIG>(j));
}

// RMSNorm(1+w) of the raw 1024-vector `hs` in shared memory, evaluated by every warp for itself: a lane reads the 32
// values of its own chunks, the warp sums the squares with one butterfly (so every warp gets the same bits), and the lane
// keeps its normalised values packed in registers -- exactly the operand consume_k1024 wants.  No block-wide reduction,
// no second trip through shared memory.
template <bool CONTIG>
__device__ __forceinline__ void norm_to_regs(const bf16* hs, const uint4 (&wn)[4], uint4 (&xq)[4]) {
    uint4 hq[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) hq[j] = *reinterpret_cast<const uint4*>(hs + lane_chunk<CONTIG>(j) * 8);
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const uint32_t w[4] = {hq[j].x, hq[j].y, hq[j].z, hq[j].w};
#pragma unroll
        for (int k = 0; k < 4; ++k) { ss = fmaf(bf_lo(w[k]), bf_lo(w[k]), ss); ss = fmaf(bf_hi(w[k]), bf_hi(w[k]), ss); }
    }
    ss = warp_sum(ss);
    const float r = rsqrt_ieee(ss * (1.0f / HIDDEN) + RMS_EPS);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const uint32_t h[4] = {hq[j].x, hq[j].y, hq[j].z, hq[j].w};
        const uint32_t w[4] = {wn[j].x, wn[j].y, wn[j].z, wn[j].w};
        uint32_t o[4];
#pragma unroll
        for (int k = 0; k < 4; ++k)
            o[k] = pack_bf16x2((bf_lo(h[k]) * r) * (1.0f + bf_lo(w[k])), (bf_hi(h[k]) * r) * (1.0f + bf_hi(w[k])));
        xq[j] = make_uint4(o[0], o[1], o[2], o[3]);
    }
}
// Split of the context over CTAs in an attention layer: chunks of >= 32 positions, CTA (kv head, chunk) owns one chunk.
struct AttGeom { int nchunk, clen, kvh, chunk, j0, j1; bool att_cta, owns_pos; };
__device__ __forceinline__ AttGeom att_geom(int pos, int b, int G) {
    AttGeom g;
    const int Lc = pos + 1;
    g.nchunk = (Lc + 31) / 32;
    { const int cap = min(ATT_MAX_CHUNKS, G / FA_KV_HEADS); if (g.nchunk > cap) g.nchunk = cap; }
    g.clen = (Lc + g.nchunk - 1) / g.nchunk;            // <= ATT_CHUNK_MAX by the host-side limit on max_seq_len
    g.att_cta = b < FA_KV_HEADS * g.nchunk;
    g.kvh = b / g.nchunk; g.chunk = b % g.nchunk;
    g.j0 = g.chunk * g.clen; g.j1 = min(Lc, g.j0 + g.clen);
    g.owns_pos = g.att_cta && pos >= g.j0 && pos < g.j1;
    return g;
}

// ------------------------------------------------------------------------------------------------
// kernel
// ------------------------------------------------------------------------------------------------
template <bool FP4>
__global__ void __launch_bounds__(STREAM_THREADS, 1) decode_stream_kernel(const DecodeArgs a) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    Smem& s = *reinterpret_cast<Smem*>(smem_raw);
    StreamWorkspace* ws = a.ws;
    const int b = blockIdx.x, G = gridDim.x;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

    if (tid == 0) s.abort_flag = (ld_volatile(&ws->err) != 0) ? 1 : 0;
    __syncthreads();
    if (s.abort_flag) return;                 // sticky error from an earlier launch: the whole CTA leaves before touching the ring
    if (tid == 0) {
        for (int i = 0; i < NSLOTS; ++i) {
            mbar_init(smem_u32(&s.full[i]), 1);
            mbar_init(smem_u32(&s.empty[i]), NCONS_WARPS);
        }
        mbar_init(smem_u32(&s.side_go), 1);
        mbar_init(smem_u32(&s.side_done), 1);
        mbar_fence_init();
    }
    if (tid < NUM_LAYERS) load_layer<FP4>(a.layers, tid, s.layers[tid]);
    if (tid >= 32 && tid < 32 + PT_COUNT) {
        const int i = tid - 32;
        constexpr int n_of[PT_COUNT / 2] = {TILES_A_DN, TILES_A_FA, TILES_C, UNITS_D, TILES_E, DN_V_SIZE / 2, DN_CONV_CH / 2, TILES_LM, FP4_LM_BLOCKS};
        s.pt[i] = part_begin(n_of[i >> 1], b + (i & 1), G);
    }
    if (tid >= 64 && tid < 64 + 256 && tid - 64 < G) s.lm_row0[tid - 64] = FP4 ? part_begin(FP4_LM_BLOCKS, tid - 64, G) * 128 : part_begin(TILES_LM, tid - 64, G) * 8;
    __syncthreads();

    Abort ab{&s.abort_flag, &ws->err};
    Ring ring{smem_u32(s.ring), smem_u32(s.full), smem_u32(s.empty), 0u};

    if (warp == NCONS_WARPS) {
        if (lane == 0) produce<FP4>(a, s, ring, ab);
        __syncwarp();
    } else if (warp == NCONS_WARPS + 1) {
        // ---- service warp: memory updates that need a fence, taken off the consumers' path ----
        // DeltaNet layer: the conv-window shift of this CTA's channel pairs.  Once the consumers have read all of `o`, every
        // CTA has finished the layer's stage B and nobody reads the old window any more.
        // Attention layer: the CTA whose chunk holds the current position appends the new K / V row to the cache (the
        // consumers use the copies in shared memory for this token).
        // A fence that orders such stores before this CTA's next publication costs more than a microsecond; here it delays
        // nobody: the consumers only check, just before they publish the layer's output, that it has completed.
        const int n_layers = a.dbg_num_layers > 0 ? a.dbg_num_layers : NUM_LAYERS;
        unsigned n_side = 0;
        for (int step = 0; step < a.n_steps; ++step) {
            int i_dn = 0, i_fa = 0;
            const int pos = a.position + step;
            for (int layer = 0; layer < n_layers; ++layer, ++n_side) {
                const unsigned ep = epoch_of(a, step, layer);
                mbar_wait(smem_u32(&s.side_go), n_side & 1u, ab);
                bool stored = false;
                if (s.layers[layer].type == 0) {
                    float* conv = a.conv_bufs + (size_t)i_dn * DN_CONV_CH * 4;
                    for (int c = s.pt[PT_CS0] + lane; c < s.pt[PT_CS1]; c += 32) {
                        const uint32_t xw = poll_word(&ws->xa[c], ep, ab);
                        const float4 c0 = ld_cg(reinterpret_cast<const float4*>(conv) + 2 * c);
                        const float4 c1 = ld_cg(reinterpret_cast<const float4*>(conv) + 2 * c + 1);
                        reinterpret_cast<float4*>(conv)[2 * c] = make_float4(c0.y, c0.z, c0.w, bf_lo(xw));
                        reinterpret_cast<float4*>(conv)[2 * c + 1] = make_float4(c1.y, c1.z, c1.w, bf_hi(xw));
                        stored = true;
                    }
                    ++i_dn;
                } else {
                    const AttGeom ag = att_geom(pos, b, G);
                    if (ag.owns_pos) {
                        const size_t row = ((size_t)i_fa * FA_KV_HEADS + ag.kvh) * a.max_seq_len + pos;
                        uint32_t* krow = reinterpret_cast<uint32_t*>(a.k_cache + row * FA_HEAD_DIM);
                        uint32_t* vrow = reinterpret_cast<uint32_t*>(a.v_cache + row * FA_HEAD_DIM);
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            const int wd = lane + 32 * i;
                            krow[wd] = pack_bf16x2(s.kcur[2 * wd], s.kcur[2 * wd + 1]);
                            vrow[wd] = s.vcur[wd];
                        }
                        stored = true;
                    }
                    ++i_fa;
                }
                if (stored) __threadfence();
                __syncwarp();
                if (lane == 0) mbar_arrive(smem_u32(&s.side_done), 1);
            }
        }
    } else {
        // =========================== consumers ===========================
        int tok = a.token_in ? __ldg(a.token_in) : a.token_imm;
        const int n_layers = a.dbg_num_layers > 0 ? a.dbg_num_layers : NUM_LAYERS;
        unsigned n_side = 0;                      // layers finished so far (phase of the two service-warp barriers)
        for (int step = 0; step < a.n_steps; ++step) {
            if (a.forced_ids) tok = __ldg(a.forced_ids + step);
            if (tok < 0 || tok >= VOCAB) { if (tid == 0) atomicCAS(&ws->err, 0, (int)ERR_BAD_ARG); tok = 0; }
            const int pos = a.position + step;
            const bool last_step = (step == a.n_steps - 1);
            int i_dn = 0, i_fa = 0;

            for (int layer = 0; layer < n_layers; ++layer) {
                const LayerW& L = s.layers[layer];
                const int stamp_row = layer;
                Q35_STAMP(0);
                const unsigned ep = epoch_of(a, step, layer);
                const bool dn = (L.type == 0);
                bool att_owner = false;                    // attention layer: this CTA's chunk holds the current position
                const bf16* w_post = (const bf16*)L.p[W_POST_NORM];

                // ---- DeltaNet: issue the state / conv loads of stage B before any waiting ----
                const int pp0 = s.pt[PT_PAIR0], pp1 = s.pt[PT_PAIR1];   // value-row pairs
                float4 st0 = make_float4(0, 0, 0, 0), st1 = st0, cv0 = st0, cv1 = st0;
                float* conv = a.conv_bufs + (size_t)i_dn * DN_CONV_CH * 4;
                float* state = a.dn_states + (size_t)i_dn * DN_HEADS * DN_V * DN_K;
                const int my_pair = pp0 + warp;                     // at most one pair per warp when G >= 64
                if (dn && my_pair < pp1) {
                    const int r0 = 2 * my_pair;                     // rows r0, r0+1 of head r0 >> 7
                    st0 = ld_cg(reinterpret_cast<const float4*>(state + (size_t)r0 * DN_K) + lane);
                    st1 = ld_cg(reinterpret_cast<const float4*>(state + (size_t)(r0 + 1) * DN_K) + lane);
                    cv0 = ld_cg(reinterpret_cast<const float4*>(conv) + 2 * DN_QK_SIZE + r0);
                    cv1 = ld_cg(reinterpret_cast<const float4*>(conv) + 2 * DN_QK_SIZE + r0 + 1);
                }

                // ================= stage A: input norm + fused projection =================
                {
                    uint4 wn[4], xq[4];
                    load_lane_chunks<FP4>((const bf16*)L.p[W_IN_NORM], wn);     // in flight while the input is awaited
                    if (layer == 0) reinterpret_cast<uint32_t*>(s.h)[tid] = __ldg(reinterpret_cast<const uint32_t*>(a.embed + (size_t)tok * HIDDEN) + tid);
                    else if (a.dbg_teacher) reinterpret_cast<uint32_t*>(s.h)[tid] = __ldg(reinterpret_cast<const uint32_t*>(a.dbg_teacher + layer * HIDDEN) + tid);
                    else fetch_vec1024(ws->h2, epoch_of(a, step, layer - 1), s.h, ab);
                    cons_sync();
                    norm_to_regs<FP4>(s.h, wn, xq);
                    Q35_STAMP(1);
                    const int u0 = s.pt[dn ? PT_A_DN0 : PT_A_FA0], u1 = s.pt[dn ? PT_A_DN1 : PT_A_FA1];
                    bf16* stage_h = reinterpret_cast<bf16*>(s.stage);
                    if (FP4) {
                        // qkv / z (or q, k, v) tiles are NVFP4; the 16+16 rows of the b and a projections stay bf16
                        const int n_q = dn ? max(0, min(u1, (DN_CONV_CH + DN_V_SIZE) / 8) - u0) : (u1 - u0);
                        consume_k1024_fp4<1>(ring, n_q, xq, ab, [&](int row, const float (&acc)[1]) { stage_h[row] = f2bf(acc[0]); });
                        if (u1 - u0 > n_q) {
                            // the few CTAs that own bf16 rows of this stage need the activations in the interleaved split too
                            uint4 wi[4], xi[4];
                            load_lane_chunks<false>((const bf16*)L.p[W_IN_NORM], wi);
                            norm_to_regs<false>(s.h, wi, xi);
                            consume_k1024<1>(ring, u1 - u0 - n_q, xi, ab, [&](int row, const float (&acc)[1]) { stage_h[n_q * 8 + row] = f2bf(acc[0]); });
                        }
                    } else {
                        consume_k1024<1>(ring, u1 - u0, xq, ab, [&](int row, const float (&acc)[1]) { stage_h[row] = f2bf(acc[0]); });
                    }
                    Q35_STAMP(10);
                    // one coalesced store per CTA: a line that is written once reaches its pollers fastest
                    cons_sync();
                    if (tid < (u1 - u0) * 4) st_word(&ws->xa[u0 * 4 + tid], s.stage[tid], ep);
                }

                Q35_STAMP_ALL(2);
                if (dn) {
                    // ================= stage B (DeltaNet): conv, norms, recurrence =================
                    const bf16* conv_w = (const bf16*)L.p[W_CONV];
                    const int hlo = (2 * pp0) >> 7, hhi = (pp1 > pp0) ? ((2 * pp1 - 1) >> 7) : hlo;   // at most two heads per CTA
                    uint32_t vw_pre = 0;
                    {
                        // 256 threads: slot (head) x {q,k} x 64 words of two channels
                        const int slot = tid >> 7, isk = (tid >> 6) & 1, wi = tid & 63;
                        const bool act = tid < 256 && (pp1 > pp0) && (hlo + slot <= hhi);
                        float c0 = 0.f, c1 = 0.f, sq = 0.f;
                        if (act) {
                            const int ch = isk * DN_QK_SIZE + (hlo + slot) * DN_K + 2 * wi;
                            const float4 s0 = ld_cg(reinterpret_cast<const float4*>(conv) + ch);
                            const float4 s1 = ld_cg(reinterpret_cast<const float4*>(conv) + ch + 1);
                            const uint32_t xw = poll_word(&ws->xa[ch >> 1], ep, ab);
                            c0 = conv_silu(conv_w, ch, s0, bf_lo(xw));
                            c1 = conv_silu(conv_w, ch + 1, s1, bf_hi(xw));
                            sq = rbf(c0 * c0) + rbf(c1 * c1);
                        }
                        if (my_pair < pp1) vw_pre = poll_word(&ws->xa[(2 * DN_QK_SIZE + 2 * my_pair) >> 1], ep, ab);
                        const float wsum = warp_sum(sq);
                        cons_sync();
                        Q35_STAMP(11);
                        if (lane == 0) s.red[warp] = wsum;
                        cons_sync();
                        if (act) {
                            float tot = s.red[warp & ~1] + s.red[warp | 1];
                            tot = rbf(tot);
                            tot = rbf(tot + 1e-6f);
                            // torch's CPU rsqrt on a 16-element bf16 tensor takes the scalar path, which rounds
                            // sqrt to bf16 before the reciprocal; decode mirrors that.
                            const float inv = rbf(1.0f / rbf(sqrtf(tot)));
                            float n0 = rbf(c0 * inv), n1 = rbf(c1 * inv);
                            if (!isk) { n0 *= 0.08838834764831845f; n1 *= 0.08838834764831845f; }   // q * 1/sqrt(128) in f32
                            s.qk[slot][isk][2 * wi] = n0;
                            s.qk[slot][isk][2 * wi + 1] = n1;
                        }
                        if (tid >= 256 && tid < 258 && (pp1 > pp0) && hlo + (tid - 256) <= hhi) {
                            const int sl = tid - 256, h = hlo + sl;
                            const uint32_t bw = poll_word(&ws->xa[(DN_CONV_CH + DN_V_SIZE + h) >> 1], ep, ab);
                            const uint32_t aw = poll_word(&ws->xa[(DN_CONV_CH + DN_V_SIZE + DN_HEADS + h) >> 1], ep, ab);
                            const float bb = (h & 1) ? bf_hi(bw) : bf_lo(bw);
                            const float aa = (h & 1) ? bf_hi(aw) : bf_lo(aw);
                            const float x = aa + bf2f(((const bf16*)L.p[W_DTBIAS])[h]);
                            const float sp = (x > 20.f) ? x : log1pf(expf(x));
                            const float g = -expf(bf2f(((const bf16*)L.p[W_ALOG])[h])) * sp;
                            s.hd[sl][0] = rbf(sigmoid_f(bb));
                            s.hd[sl][1] = expf(g);
                        }
                        cons_sync();
                    }
                    if (my_pair < pp1) {
                        const int r0 = 2 * my_pair, h = r0 >> 7, slot = h - hlo;
                        const float4 q4 = *reinterpret_cast<const float4*>(&s.qk[slot][0][lane * 4]);
                        const float4 k4 = *reinterpret_cast<const float4*>(&s.qk[slot][1][lane * 4]);
                        const float beta = s.hd[slot][0], decay = s.hd[slot][1];
                        const int ch = 2 * DN_QK_SIZE + r0;
                        const uint32_t vw = vw_pre;
                        const float vv[2] = {conv_silu(conv_w, ch, cv0, bf_lo(vw)), conv_silu(conv_w, ch + 1, cv1, bf_hi(vw))};
                        float4 sv[2] = {st0, st1};
                        float ov[2];
#pragma unroll
                        for (int r = 0; r < 2; ++r) {
                            float4 t = sv[r];
                            t.x = __fmul_rn(t.x, decay); t.y = __fmul_rn(t.y, decay); t.z = __fmul_rn(t.z, decay); t.w = __fmul_rn(t.w, decay);
                            float kv = __fadd_rn(__fadd_rn(__fadd_rn(__fmul_rn(t.x, k4.x), __fmul_rn(t.y, k4.y)), __fmul_rn(t.z, k4.z)), __fmul_rn(t.w, k4.w));
                            kv = warp_sum(kv);
                            const float delta = __fmul_rn(__fsub_rn(vv[r], kv), beta);
                            t.x = __fadd_rn(t.x, __fmul_rn(k4.x, delta)); t.y = __fadd_rn(t.y, __fmul_rn(k4.y, delta));
                            t.z = __fadd_rn(t.z, __fmul_rn(k4.z, delta)); t.w = __fadd_rn(t.w, __fmul_rn(k4.w, delta));
                            float o = __fadd_rn(__fadd_rn(__fadd_rn(__fmul_rn(t.x, q4.x), __fmul_rn(t.y, q4.y)), __fmul_rn(t.z, q4.z)), __fmul_rn(t.w, q4.w));
                            ov[r] = warp_sum(o);
                            reinterpret_cast<float4*>(state + (size_t)(r0 + r) * DN_K)[lane] = t;
                        }
                        if (lane == 0) s.stage_b[warp] = pack_bf16x2(ov[0], ov[1]);
                    }
                    cons_sync();
                    if (tid < pp1 - pp0) st_word(&ws->o[pp0 + tid], s.stage_b[tid], ep);

                    Q35_STAMP(3);
                    // ================= stage C (DeltaNet): gated norm (one head per warp) =================
                    {
                        const int h = warp;
                        // z was published in stage A, long ago: everything that depends on z alone is done before `o` is awaited
                        const u64* po = &ws->o[h * 64 + lane * 2];
                        const u64* pz = &ws->xa[(DN_CONV_CH >> 1) + h * 64 + lane * 2];
                        const uint2 nrw = __ldg(reinterpret_cast<const uint2*>(L.p[W_GNORM]) + lane);
                        uint32_t z0, z1, o0, o1;
                        poll2(pz, pz + 1, ep, ab, z0, z1);
                        const float sz[4] = {silu_f(bf_lo(z0)), silu_f(bf_hi(z0)), silu_f(bf_lo(z1)), silu_f(bf_hi(z1))};
                        const float nw[4] = {bf_lo(nrw.x), bf_hi(nrw.x), bf_lo(nrw.y), bf_hi(nrw.y)};
                        poll2(po, po + 1, ep, ab, o0, o1);
                        const float ov[4] = {bf_lo(o0), bf_hi(o0), bf_lo(o1), bf_hi(o1)};
                        const float var = warp_sum(ov[0] * ov[0] + ov[1] * ov[1] + ov[2] * ov[2] + ov[3] * ov[3]) * (1.0f / DN_V);
                        const float r = rsqrt_ieee(var + RMS_EPS);
                        uint32_t out[2];
#pragma unroll
                        for (int i = 0; i < 2; ++i) {
                            const float t0 = rbf(nw[2 * i] * rbf(ov[2 * i] * r)), t1 = rbf(nw[2 * i + 1] * rbf(ov[2 * i + 1] * r));
                            out[i] = pack_bf16x2(t0 * sz[2 * i], t1 * sz[2 * i + 1]);
                        }
                        *reinterpret_cast<uint2*>(s.x + h * DN_V + lane * 4) = make_uint2(out[0], out[1]);
                    }
                    ++i_dn;
                } else {
                    // ================= attention: B1 scores + chunk statistics, B2 P.V partials, B3 merge + gate =================
                    // The context is split into chunks of >= 32 positions; CTA (kv head, chunk) owns one chunk.
                    bf16* kc = a.k_cache + (size_t)i_fa * FA_KV_HEADS * a.max_seq_len * FA_HEAD_DIM;
                    bf16* vc = a.v_cache + (size_t)i_fa * FA_KV_HEADS * a.max_seq_len * FA_HEAD_DIM;
                    const AttGeom ag = att_geom(pos, b, G);
                    const int nchunk = ag.nchunk, kvh = ag.kvh, chunk = ag.chunk, j0 = ag.j0, j1 = ag.j1;
                    const bool att_cta = ag.att_cta;
                    att_owner = ag.owns_pos;
                    if (att_cta) {
                        // this warp's first two key rows do not depend on the current token: request them before the q / k / v of
                        // the token are awaited, so their L2 latency runs under the hand-off
                        uint4 k_pre_a = make_uint4(0, 0, 0, 0), k_pre_b = k_pre_a;
                        {
                            const int j = j0 + warp, jb = j + NCONS_WARPS;
                            if (j < j1 && j != pos) k_pre_a = ld_cg(reinterpret_cast<const uint4*>(kc + ((size_t)kvh * a.max_seq_len + j) * FA_HEAD_DIM) + lane);
                            if (jb < j1 && jb != pos) k_pre_b = ld_cg(reinterpret_cast<const uint4*>(kc + ((size_t)kvh * a.max_seq_len + jb) * FA_HEAD_DIM) + lane);
                        }
                        if (warp < FA_GQA + 1) {
                            // warps 0..3: the four query heads of this kv head; warp 4: the new key.
                            // lane l holds elements {2l, 2l+1} + 64*i, i = 0..3 (four flagged words)
                            const bool isq = warp < FA_GQA;
                            const int e0 = isq ? (kvh * FA_GQA + warp) * 2 * FA_HEAD_DIM : FA_QPROJ + kvh * FA_HEAD_DIM;
                            const bf16* nw = (const bf16*)(isq ? L.p[W_QNORM] : L.p[W_KNORM]);
                            float xv[8], ss = 0.f;
                            uint32_t wv[4];
                            poll4(&ws->xa[(e0 >> 1) + lane], 32, ep, ab, wv);
#pragma unroll
                            for (int i = 0; i < 4; ++i) {
                                xv[2 * i] = bf_lo(wv[i]); xv[2 * i + 1] = bf_hi(wv[i]);
                                ss += xv[2 * i] * xv[2 * i] + xv[2 * i + 1] * xv[2 * i + 1];
                            }
                            const float r = rsqrt_ieee(warp_sum(ss) * (1.0f / FA_HEAD_DIM) + RMS_EPS);
#pragma unroll
                            for (int i = 0; i < 4; ++i) {
                                const int d = 2 * lane + 64 * i;
                                xv[2 * i] = rbf((xv[2 * i] * r) * (1.0f + bf2f(nw[d])));
                                xv[2 * i + 1] = rbf((xv[2 * i + 1] * r) * (1.0f + bf2f(nw[d + 1])));
                            }
                            // RoPE on dims [0,64): pairs (d, d+32).  Lanes 0-15 hold dims 2l,2l+1; lanes 16-31 hold 32+2(l-16), +1.
                            {
                                const int fi = 2 * (lane & 15);
                                const float ang0 = (float)pos * c_rope_inv_freq[fi], ang1 = (float)pos * c_rope_inv_freq[fi + 1];
                                const float c0 = rbf(cosf(ang0)), s0 = rbf(sinf(ang0)), c1 = rbf(cosf(ang1)), s1 = rbf(sinf(ang1));
                                const float p0 = __shfl_xor_sync(0xffffffffu, xv[0], 16), p1 = __shfl_xor_sync(0xffffffffu, xv[1], 16);
                                if (lane < 16) {   // own = x1, partner = x2
                                    xv[0] = rbf(rbf(xv[0] * c0) + rbf(-p0 * s0));
                                    xv[1] = rbf(rbf(xv[1] * c1) + rbf(-p1 * s1));
                                } else {           // own = x2, partner = x1
                                    xv[0] = rbf(rbf(xv[0] * c0) + rbf(p0 * s0));
                                    xv[1] = rbf(rbf(xv[1] * c1) + rbf(p1 * s1));
                                }
                            }
                            float* dst = isq ? s.q[warp] : s.kcur;
#pragma unroll
                            for (int i = 0; i < 4; ++i) { dst[2 * lane + 64 * i] = xv[2 * i]; dst[2 * lane + 64 * i + 1] = xv[2 * i + 1]; }
                        } else if (warp == FA_GQA + 1 && ag.owns_pos) {
                            // the new value row stays in shared memory for this token; the service warp appends it (and the
                            // key row from kcur) to the cache
                            uint32_t wv[4];
                            poll4(&ws->xa[((FA_QPROJ + FA_KV_SIZE + kvh * FA_HEAD_DIM) >> 1) + lane], 32, ep, ab, wv);
#pragma unroll
                            for (int i = 0; i < 4; ++i) s.vcur[lane + 32 * i] = wv[i];
                        }
                        cons_sync();
                        if (ag.owns_pos && tid == 0) { mbar_arrive(smem_u32(&s.side_go), 1); }
                        // ---- scores of this chunk, two positions per warp in flight ----
                        {
                            float qr[FA_GQA][8];
#pragma unroll
                            for (int g = 0; g < FA_GQA; ++g)
#pragma unroll
                                for (int i = 0; i < 8; ++i) qr[g][i] = s.q[g][lane * 8 + i];
                            for (int j = j0 + warp; j < j1; j += 2 * NCONS_WARPS) {
                                const int jb = j + NCONS_WARPS;
                                uint4 ka = k_pre_a, kb = k_pre_b;
                                if (j != j0 + warp) {          // later rounds of a long chunk
                                    ka = make_uint4(0, 0, 0, 0); kb = ka;
                                    if (j != pos) ka = ld_cg(reinterpret_cast<const uint4*>(kc + ((size_t)kvh * a.max_seq_len + j) * FA_HEAD_DIM) + lane);
                                    if (jb < j1 && jb != pos) kb = ld_cg(reinterpret_cast<const uint4*>(kc + ((size_t)kvh * a.max_seq_len + jb) * FA_HEAD_DIM) + lane);
                                }
#pragma unroll
                                for (int r = 0; r < 2; ++r) {
                                    const int jj = r ? jb : j;
                                    if (jj >= j1) break;
                                    float kf[8];
                                    if (jj == pos) {
#pragma unroll
                                        for (int i = 0; i < 8; ++i) kf[i] = s.kcur[lane * 8 + i];
                                    } else {
                                        unpack8(r ? kb : ka, kf);
                                    }
#pragma unroll
                                    for (int g = 0; g < FA_GQA; ++g) {
                                        float d = 0.f;
#pragma unroll
                                        for (int i = 0; i < 8; ++i) d = fmaf(qr[g][i], kf[i], d);
                                        d = warp_sum(d);
                                        if (lane == 0) s.p[g][jj - j0] = rbf(d) * 0.0625f;
                                    }
                                }
                            }
                        }
                        cons_sync();
                        // ---- chunk statistics -> everyone; global max / normaliser from all chunks ----
                        const int cn = j1 - j0;
                        if (warp < FA_GQA) {
                            float mx = -INFINITY;
                            for (int j = lane; j < cn; j += 32) mx = fmaxf(mx, s.p[warp][j]);
                            mx = warp_max(mx);
                            float sm = 0.f;
                            for (int j = lane; j < cn; j += 32) sm += expf(s.p[warp][j] - mx);
                            sm = warp_sum(sm);
                            if (lane == 0) {
                                st_word(&ws->att_stat[kvh * FA_GQA + warp][chunk][0], __float_as_uint(mx), ep);
                                st_word(&ws->att_stat[kvh * FA_GQA + warp][chunk][1], __float_as_uint(sm), ep);
                            }
                        }
                        if (tid < nchunk * FA_GQA * 2) {
                            const int g = tid / (nchunk * 2), r = tid % (nchunk * 2);
                            s.part[g * (2 * ATT_MAX_CHUNKS) + r] = __uint_as_float(poll_word(&ws->att_stat[kvh * FA_GQA + g][0][0] + r, ep, ab));
                        }
                        cons_sync();
                        if (warp < FA_GQA) {
                            const float* st = &s.part[warp * (2 * ATT_MAX_CHUNKS)];
                            float mx = -INFINITY;
                            for (int c = lane; c < nchunk; c += 32) mx = fmaxf(mx, st[2 * c]);
                            mx = warp_max(mx);
                            float sm = 0.f;
                            for (int c = lane; c < nchunk; c += 32) sm += st[2 * c + 1] * expf(st[2 * c] - mx);
                            sm = warp_sum(sm);
                            if (lane == 0) { s.ml[warp][0] = mx; s.ml[warp][1] = sm; }
                        }
                        cons_sync();
                        for (int i = tid; i < FA_GQA * cn; i += NCONS) {
                            const int gg = i / cn, jj = i % cn;
                            s.p[gg][jj] = rbf(expf(s.p[gg][jj] - s.ml[gg][0]) / s.ml[gg][1]);
                        }
                        cons_sync();
                        // ---- P.V over this chunk: 4 heads x 128 threads, 2 dims each, 8 value rows in flight ----
                        {
                            const int g = tid >> 7, d2 = tid & 127;
                            float acc0 = 0.f, acc1 = 0.f;
                            const uint32_t* vb = reinterpret_cast<const uint32_t*>(vc + ((size_t)kvh * a.max_seq_len + j0) * FA_HEAD_DIM) + d2;
                            // 32 value rows in flight: a chunk of up to 32 positions (every context below 2368 tokens)
                            // costs one L2 round trip, not four
                            for (int jj = 0; jj < cn; jj += 32) {
                                uint32_t vr[32];
#pragma unroll
                                for (int u = 0; u < 32; ++u)
                                    vr[u] = (jj + u >= cn) ? 0u : (j0 + jj + u == pos) ? s.vcur[d2] : ld_cg(vb + (size_t)(jj + u) * (FA_HEAD_DIM / 2));
#pragma unroll
                                for (int u = 0; u < 32; ++u) {
                                    const float p = (jj + u < cn) ? s.p[g][jj + u] : 0.f;
                                    acc0 = fmaf(p, bf_lo(vr[u]), acc0);
                                    acc1 = fmaf(p, bf_hi(vr[u]), acc1);
                                }
                            }
                            // the partial travels as flagged words like every other hand-off: no fence, no separate flag
                            st_word(&ws->att_part[chunk][kvh * FA_GQA + g][2 * d2], __float_as_uint(acc0), ep);
                            st_word(&ws->att_part[chunk][kvh * FA_GQA + g][2 * d2 + 1], __float_as_uint(acc1), ep);
                        }
                    }
                    // ---- B3: CTA h < 8 merges the partials of query head h and applies the sigmoid gate ----
                    if (b < FA_Q_HEADS) {
                        const int qh = b;
                        cons_sync();                      // P of this CTA's chunk (s.p) is no longer needed: it holds the group sums now
                        {
                            // 4 groups of 128 threads: group q sums chunks q, q+4, ... in ascending order, two dims per thread,
                            // four chunks (8 flagged words) in flight per round trip
                            const int d = tid & 127, grp = tid >> 7;
                            float a0 = 0.f, a1 = 0.f;
                            for (int c0 = grp; c0 < nchunk; c0 += 16) {
                                uint32_t w[8];
                                poll_pairs<4>(&ws->att_part[c0][qh][2 * d], 4 * FA_Q_HEADS * FA_HEAD_DIM, (nchunk - c0 + 3) / 4, ep, ab, w);
#pragma unroll
                                for (int u = 0; u < 4; ++u) { a0 += __uint_as_float(w[2 * u]); a1 += __uint_as_float(w[2 * u + 1]); }
                            }
                            reinterpret_cast<float2*>(&s.p[0][0])[grp * 128 + d] = make_float2(a0, a1);
                        }
                        cons_sync();
                        if (tid < 128) {
                            const int d = 2 * tid;
                            const int ge = qh * 2 * FA_HEAD_DIM + FA_HEAD_DIM + d;
                            const uint32_t gw = poll_word(&ws->xa[ge >> 1], ep, ab);
                            float2 acc = make_float2(0.f, 0.f);
#pragma unroll
                            for (int q = 0; q < 4; ++q) {
                                const float2 v = reinterpret_cast<const float2*>(&s.p[0][0])[q * 128 + tid];
                                acc.x += v.x; acc.y += v.y;
                            }
                            const float u0 = rbf(acc.x) * rbf(sigmoid_f(bf_lo(gw))), u1 = rbf(acc.y) * rbf(sigmoid_f(bf_hi(gw)));
                            st_word(&ws->o[(qh * FA_HEAD_DIM + d) >> 1], pack_bf16x2(u0, u1), ep);
                        }
                    }
                    Q35_STAMP(3);
                    // ---- stage C (attention): the gated attention output is the GEMV input ----
                    {
                        uint32_t w0, w1;
                        poll2(&ws->o[tid], &ws->o[tid + NCONS], ep, ab, w0, w1);
                        reinterpret_cast<uint32_t*>(s.x)[tid] = w0;
                        reinterpret_cast<uint32_t*>(s.x)[tid + NCONS] = w1;
                    }
                    ++i_fa;
                }
                cons_sync();
                // DeltaNet: every warp has its head's `o`, so all CTAs are past stage B.  Attention: the CTA that holds the new
                // K / V row has signalled already, the others have no side work.
                if (tid == 0 && (dn || !att_owner)) mbar_arrive(smem_u32(&s.side_go), 1);
                Q35_STAMP(4);
                // ---- stage C tail: output projection (K = 2048, 4 rows per tile) + residual ----
                {
                    const bf16* hin = s.h;
                    const int u0 = s.pt[PT_C0], nt = s.pt[PT_C1] - u0;
                    if (FP4) {
                        // 4 rows x 1024 bytes of nibbles per tile, two tiles at a time: warp = (tile w/8, row (w/2)%4, K half w%2), 32
                        // groups of 32 per half row, one per lane
                        float x[32];
                        load_x32(s.x, (warp & 1) * 1024 + 32 * lane, x);
                        const uint32_t row = (uint32_t)((warp >> 1) & 3), half = (uint32_t)(warp & 1);
                        for (int tb = 0; tb < nt; tb += 2) {
                            const int ti = tb + (warp >> 3);
                            if (ti < nt) {
                                const unsigned tile = ring.t + (unsigned)ti;
                                mbar_wait(ring.full_bar(tile), ring.phase(tile), ab);
                                const uint4 pk = lds128(ring.slot_addr(tile) + row * 1024u + half * 512u + (uint32_t)lane * 16u);
                                const float sc = lds_half(ring.slot_addr(tile) + FP4_SCALE_OFF + row * 128u + (half * 32u + (uint32_t)lane) * 2u);
                                const float acc = warp_sum(dot32_fp4(pk, x) * sc);
                                if (lane == 0) {
                                    s.part[ti * 16 + row * 4 + half] = acc;
                                    s.part[ti * 16 + row * 4 + 2 + half] = 0.f;
                                    mbar_arrive(ring.empty_bar(tile), 2);
                                }
                            }
                        }
                    } else {
                    // two tiles at a time: warp = (tile w/8, row (w/2)%4, K half w%2), so a CTA with two tiles (most have one
                    // or two) is done as soon as a CTA with one
                    const int crow = (warp >> 1) & 3, chalf = warp & 1;
                    uint4 xc[4];
#pragma unroll
                    for (int j = 0; j < 4; ++j) xc[j] = *reinterpret_cast<const uint4*>(s.x + chalf * 1024 + (j * 32 + lane) * 8);
                    for (int tb = 0; tb < nt; tb += 2) {
                        const int ti = tb + (warp >> 3);
                        if (ti < nt) {
                            const unsigned tile = ring.t + (unsigned)ti;
                            mbar_wait(ring.full_bar(tile), ring.phase(tile), ab);
                            const uint32_t base = ring.slot_addr(tile) + (uint32_t)crow * 4096u + (uint32_t)chalf * 2048u + (uint32_t)lane * 16u;
                            uint4 wq[4];
#pragma unroll
                            for (int j = 0; j < 4; ++j) wq[j] = lds128(base + j * 512);
                            const float a0 = dot8m(wq[2], xc[2], dot8m(wq[0], xc[0], 0.f)), a1 = dot8m(wq[3], xc[3], dot8m(wq[1], xc[1], 0.f));
                            const float acc = warp_sum(a0 + a1);
                            if (lane == 0) { s.part[ti * 16 + crow * 2 + chalf] = acc; mbar_arrive(ring.empty_bar(tile), 2); }
                        }
                    }
                    }
                    ring.t += (unsigned)nt;
                    cons_sync();
                    if (tid < nt * 2) {
                        const int ti = tid >> 1, pr = tid & 1;
                        // partial sums of rows 2 pr and 2 pr + 1: NVFP4 keeps four slots per row, bf16 one per K half
                        const float* pp = &s.part[ti * 16 + pr * (FP4 ? 8 : 4)];
                        const float y0 = FP4 ? ((pp[0] + pp[1]) + pp[2]) + pp[3] : pp[0] + pp[1];
                        const float y1 = FP4 ? ((pp[4] + pp[5]) + pp[6]) + pp[7] : pp[2] + pp[3];
                        const int row = (u0 + ti) * 4 + 2 * pr;
                        st_word(&ws->h1[row >> 1], pack_bf16x2(bf2f(hin[row]) + rbf(y0), bf2f(hin[row + 1]) + rbf(y1)), ep);
                    }
                }

                Q35_STAMP_ALL(5);
                // ================= stage D: post norm, gate/up with SiLU*up =================
                {
                    uint4 wn[4], xq[4];
                    load_lane_chunks<FP4>(w_post, wn);
                    fetch_vec1024(ws->h1, ep, s.h1, ab);
                    cons_sync();
                    norm_to_regs<FP4>(s.h1, wn, xq);
                    Q35_STAMP(6);
                    const int u0 = s.pt[PT_D0], u1 = s.pt[PT_D1];
                    bf16* stage_h = reinterpret_cast<bf16*>(s.stage);
                    auto epi_d = [&](int row, const float (&acc)[2]) {
                        stage_h[row] = f2bf(rbf(silu_f(rbf(acc[0]))) * rbf(acc[1]));
                    };
                    if (FP4) {
                        consume_k1024_fp4<2>(ring, u1 - u0, xq, ab, epi_d);
                    } else {
                        consume_k1024<2>(ring, u1 - u0, xq, ab, epi_d);
                    }
                    cons_sync();
                    if (tid < (u1 - u0) * 4) st_word(&ws->m[u0 * 4 + tid], s.stage[tid], ep);
                }
                Q35_STAMP_ALL(7);
                // ================= stage E: down projection (K = 3584, 2 rows per tile) + residual =================
                {
                    {
                        // 1792 words: 3 per thread + one more for the first half of the threads
                        uint32_t mv[4];
                        const int nw = (tid + 3 * NCONS < INTER / 2) ? 4 : 3;
                        poll_n<4>(&ws->m[tid], NCONS, nw, ep, ab, mv);
#pragma unroll
                        for (int i = 0; i < 4; ++i) if (i < nw) reinterpret_cast<uint32_t*>(s.x)[tid + i * NCONS] = mv[i];
                    }
                    cons_sync();
                    Q35_STAMP(8);
                    const int u0 = s.pt[PT_E0], nt = s.pt[PT_E1] - u0;
                    if (FP4) {
                        // 2 rows x 1792 bytes of nibbles per tile; warp: tile w/4, row (w%4)/2, K half w%2 = 56 groups of 32:
                        // lane l takes group l and, for l < 24, group 32 + l
                        const int half = warp & 1;
                        for (int g = 0; g < nt; g += 4) {
                            const int ti = g + (warp >> 2);
                            if (ti < nt) {
                                const unsigned tile = ring.t + (unsigned)ti;
                                mbar_wait(ring.full_bar(tile), ring.phase(tile), ab);
                                const uint32_t row = (uint32_t)((warp & 3) >> 1);
                                const uint32_t pb = ring.slot_addr(tile) + row * 1792u + (uint32_t)half * 896u + (uint32_t)lane * 16u;
                                const uint32_t sb = ring.slot_addr(tile) + FP4_SCALE_OFF + row * 224u + ((uint32_t)half * 56u + (uint32_t)lane) * 2u;
                                float x[32];          // a CTA owns at most four of these tiles, so each warp runs this once per stage
                                load_x32(s.x, half * 1792 + 32 * lane, x);
                                float acc = dot32_fp4(lds128(pb), x) * lds_half(sb);
                                if (lane < 24) {
                                    load_x32(s.x, half * 1792 + 32 * (32 + lane), x);
                                    acc += dot32_fp4(lds128(pb + 512), x) * lds_half(sb + 64);
                                }
                                acc = warp_sum(acc);
                                if (lane == 0) { s.part[ti * 4 + (warp & 3)] = acc; mbar_arrive(ring.empty_bar(tile), 4); }
                            }
                        }
                    } else {
                    uint4 xp[7];
#pragma unroll
                    for (int j = 0; j < 7; ++j) xp[j] = *reinterpret_cast<const uint4*>(s.x + (warp & 1) * 1792 + (j * 32 + lane) * 8);
                    for (int g = 0; g < nt; g += 4) {
                        const int ti = g + (warp >> 2);
                        if (ti < nt) {
                            const unsigned tile = ring.t + (unsigned)ti;
                            mbar_wait(ring.full_bar(tile), ring.phase(tile), ab);
                            const uint32_t base = ring.slot_addr(tile) + (uint32_t)((warp & 3) >> 1) * 7168u + (uint32_t)(warp & 1) * 3584u + (uint32_t)lane * 16u;
                            uint4 wq[7];
#pragma unroll
                            for (int j = 0; j < 7; ++j) wq[j] = lds128(base + j * 512);
                            float a0 = dot8m(wq[0], xp[0], 0.f), a1 = dot8m(wq[1], xp[1], 0.f), a2 = dot8m(wq[2], xp[2], 0.f);
                            a0 = dot8m(wq[3], xp[3], a0); a1 = dot8m(wq[4], xp[4], a1); a2 = dot8m(wq[5], xp[5], a2);
                            a0 = dot8m(wq[6], xp[6], a0);
                            const float acc = warp_sum((a0 + a1) + a2);
                            if (lane == 0) { s.part[ti * 4 + (warp & 3)] = acc; mbar_arrive(ring.empty_bar(tile), 4); }
                        }
                    }
                    }
                    ring.t += (unsigned)nt;
                    // the layer's output is the publication that the next token's readers of the conv window follow
                    if (tid == 0) mbar_wait(smem_u32(&s.side_done), n_side & 1u, ab);
                    ++n_side;
                    cons_sync();
                    if (tid < nt) {
                        const float y0 = s.part[tid * 4] + s.part[tid * 4 + 1], y1 = s.part[tid * 4 + 2] + s.part[tid * 4 + 3];
                        const int row = (u0 + tid) * 2;
                        const uint32_t hv = pack_bf16x2(bf2f(s.h1[row]) + rbf(y0), bf2f(s.h1[row + 1]) + rbf(y1));
                        st_word(&ws->h2[row >> 1], hv, ep);
                        if (last_step && a.dbg_hidden) reinterpret_cast<uint32_t*>(a.dbg_hidden + layer * HIDDEN)[row >> 1] = hv;
                        if (last_step && layer == n_layers - 1 && a.hidden_out) reinterpret_cast<uint32_t*>(a.hidden_out)[row >> 1] = hv;
                    }
                }
                Q35_STAMP_ALL(9);
            }

            // ================= LM head: final norm, 248320 x 1024 GEMV, arg-max =================
            if (!a.lm_last_only || last_step) {
                const unsigned ep_lm = epoch_of(a, step, 24);
                const int stamp_row = 24;
                Q35_STAMP(0);
                uint4 wn[4], xq[4];
                load_lane_chunks<FP4>(a.final_norm, wn);
                fetch_vec1024(ws->h2, epoch_of(a, step, n_layers - 1), s.h, ab);
                Q35_STAMP(1);
                cons_sync();
                norm_to_regs<FP4>(s.h, wn, xq);
                float best = -INFINITY;
                int best_i = 0x7fffffff;
                float* lg = (last_step ? a.logits_out : nullptr);
                // rows of the vocabulary owned by this CTA: [lm_row0, ...), in 8-row tiles (bf16) or 128-row blocks (NVFP4)
                const int lm_row0 = FP4 ? s.pt[PT_LMB0] * 128 : s.pt[PT_LM0] * 8;
                if (FP4) {
                    // tensor-core layout: one E4M3 scale per 16 weights, stored in 512-byte tiles of 128 rows x 4 blocks
                    float x[32];
#pragma unroll
                    for (int j = 0; j < 4; ++j) unpack8(xq[j], x + 8 * j);
                    const int B0 = s.pt[PT_LMB0], B1 = s.pt[PT_LMB1];
                    for (int blk = B0; blk < B1; ++blk) {
                        const unsigned tile_s = ring.t, tile_p = ring.t + 1u + (unsigned)(warp >> 2);
                        mbar_wait(ring.full_bar(tile_s), ring.phase(tile_s), ab);
                        mbar_wait(ring.full_bar(tile_p), ring.phase(tile_p), ab);
                        const uint32_t sp = ring.slot_addr(tile_p), ss = ring.slot_addr(tile_s);
#pragma unroll
                        for (int it = 0; it < 4; ++it) {
                            float vv[2];
#pragma unroll
                            for (int r = 0; r < 2; ++r) {
                                const uint32_t rit = (uint32_t)((warp & 3) * 8 + it * 2 + r);           // row inside the 32-row tile
                                const uint4 pk = lds128(sp + rit * 512u + (uint32_t)lane * 16u);
                                const float2 sc = lds_e4m3x2(ss + (uint32_t)(lane >> 1) * 512u + rit * 16u + (uint32_t)(warp >> 2) * 4u + (uint32_t)((2 * lane) & 3));
                                const float2 d = dot16x2_fp4(pk, x);
                                vv[r] = warp_sum(d.x * sc.x + d.y * sc.y);
                            }
                            if (lane == 0) {
                                const int r0 = blk * 128 + (warp >> 2) * 32 + (warp & 3) * 8 + it * 2;
                                const float v0 = rbf(vv[0]), v1 = rbf(vv[1]);
                                if (lg) { lg[r0] = v0; lg[r0 + 1] = v1; }
                                if (v0 > best) { best = v0; best_i = r0; }
                                if (v1 > best) { best = v1; best_i = r0 + 1; }
                            }
                        }
                        if (lane == 0) { mbar_arrive(ring.empty_bar(tile_p), 4); mbar_arrive(ring.empty_bar(tile_s), 1); }
                        ring.t += 5u;
                    }
                } else {
                    const int u0 = s.pt[PT_LM0], u1 = s.pt[PT_LM1];
                    // lane 0 sees the even rows of its warp's share, lane 16 the odd ones, each in ascending order
                    consume_k1024<1>(ring, u1 - u0, xq, ab, [&](int row, const float (&acc)[1]) {
                        const int r0 = u0 * 8 + row;
                        const float v0 = rbf(acc[0]);
                        if (lg) lg[r0] = v0;
                        if (v0 > best) { best = v0; best_i = r0; }
                    });
                    const float ob = __shfl_sync(0xffffffffu, best, 16);
                    const int oi = __shfl_sync(0xffffffffu, best_i, 16);
                    if (ob > best || (ob == best && oi < best_i)) { best = ob; best_i = oi; }
                }
                Q35_STAMP(2);
                // lane 0 of every warp holds that warp's best
                cons_sync();
                if (lane == 0) { s.part[warp] = best; reinterpret_cast<int*>(s.part)[NCONS_WARPS + warp] = best_i; }
                cons_sync();
                if (tid == 0) {
                    float bv = s.part[0]; int bi = reinterpret_cast<int*>(s.part)[NCONS_WARPS];
                    for (int w = 1; w < NCONS_WARPS; ++w) {
                        const float v = s.part[w]; const int i = reinterpret_cast<int*>(s.part)[NCONS_WARPS + w];
                        if (v > bv || (v == bv && i < bi)) { bv = v; bi = i; }
                    }
                    // bf16 value in the high half, row offset inside this CTA's range (< 2048) in the low half
                    st_word(&ws->lm[0][b], (__float_as_uint(bv) & 0xffff0000u) | (uint32_t)(bi - lm_row0), ep_lm);
                }
                if (warp == 0) {
                    constexpr int PER = 8;                               // up to 256 CTAs
                    u64 v[PER];
#pragma unroll
                    for (int k = 0; k < PER; ++k) v[k] = (lane + 32 * k < G) ? ld_word(&ws->lm[0][lane + 32 * k]) : 0ull;
                    float bv = -INFINITY; int bi = 0x7fffffff;
#pragma unroll
                    for (int k = 0; k < PER; ++k) {
                        const int c = lane + 32 * k;
                        if (c < G) {
                            const uint32_t w = ((uint32_t)(v[k] >> 32) == ep_lm) ? (uint32_t)v[k] : poll_word(&ws->lm[0][c], ep_lm, ab);
                            const float val = __uint_as_float(w & 0xffff0000u);
                            const int idx = s.lm_row0[c] + (int)(w & 0xffffu);
                            if (val > bv || (val == bv && idx < bi)) { bv = val; bi = idx; }
                        }
                    }
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1) {
                        const float v2 = __shfl_xor_sync(0xffffffffu, bv, o); const int i2 = __shfl_xor_sync(0xffffffffu, bi, o);
                        if (v2 > bv || (v2 == bv && i2 < bi)) { bv = v2; bi = i2; }
                    }
                    if (lane == 0) s.tok = bi;
                }
                cons_sync();
                Q35_STAMP(3);
                tok = s.tok;
                if (b == 0 && tid == 0) {
                    if (a.out_tokens) a.out_tokens[step] = tok;
                    if (last_step && a.out_token) *a.out_token = tok;
                }
            }
        }
    }
    __syncthreads();   // the producer has drained its copies; nothing is in flight when the CTA exits
}

}  // namespace q35

// ======================================= host side ==========================================
#include <cmath>
#include <cstdlib>
#include <mutex>

#include "runtime.h"

namespace q35 {

static void rope_table(float* t) {
    for (int i = 0; i < FA_ROT / 2; ++i) {
        const float e = (float)(2 * i) / (float)FA_ROT;
        const float p = (float)std::pow(1.0e7, (double)e);
        t[i] = 1.0f / p;
    }
}

static int decode_grid() {
    // one persistent CTA per SM; MEGAKERNEL_DECODE_BLOCKS overrides (same knob as the reference, kernel.cu:926-943)
    int g = device_sm_count();
    if (const char* s = getenv("MEGAKERNEL_DECODE_BLOCKS")) {
        const int v = atoi(s);
        if (v >= 64 && v <= g) g = v;
    }
    return g;
}

static unsigned g_epoch[64] = {};

// Scratch of qwen35_b200_decode_steps_static: lives in the module image, one copy on every device that
// loads the library, for the life of the process.  In host code this name is only a handle for
// cudaGetSymbolAddress -- it is not a device address and must never be handed to a kernel.
static __device__ __align__(256) unsigned char g_static_scratch[sizeof(StreamWorkspace)];
static StreamWorkspace* g_static_ptr[64] = {};
static unsigned g_static_epoch[64] = {};

static int tma_period() {
    static int v = -1;
    if (v < 0) {
        v = 400;
        if (const char* s = getenv("QWEN35_TMA_PERIOD")) v = atoi(s);
        if (v < 0) v = 0;
    }
    return v;
}

static int launch_decode_impl(const DecodeArgs& in, cudaStream_t stream, bool use_static = false, bool fp4 = false) {
    static std::once_flag once[64];
    static bool ready[64] = {};
    int dev = 0;
    Q35_CUDA_OK(cudaGetDevice(&dev));
    dev &= 63;
    std::call_once(once[dev], [&] {
        float t[FA_ROT / 2];
        rope_table(t);
        int nb = 0;
        int nb2 = 0;
        if (cudaMemcpyToSymbol(c_rope_inv_freq, t, sizeof(t)) == cudaSuccess &&
            cudaFuncSetAttribute(decode_stream_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(Smem)) == cudaSuccess &&
            cudaFuncSetAttribute(decode_stream_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(Smem)) == cudaSuccess &&
            cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, decode_stream_kernel<false>, STREAM_THREADS, sizeof(Smem)) == cudaSuccess && nb >= 1 &&
            cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb2, decode_stream_kernel<true>, STREAM_THREADS, sizeof(Smem)) == cudaSuccess && nb2 >= 1)
            ready[dev] = true;
    });
    if (!ready[dev]) { set_error("decode kernel cannot be made resident on this device (needs %zu bytes of shared memory)", sizeof(Smem)); return QWEN35_ERR_CUDA; }

    DecodeArgs a = in;
    if (a.n_steps <= 0) return QWEN35_OK;
    if (!a.layers || !a.embed || !a.final_norm || !a.lm_head || !a.k_cache || !a.v_cache || !a.dn_states || !a.conv_bufs) {
        set_error("null tensor pointer");
        return QWEN35_ERR_BAD_ARG;
    }
    if (a.position < 0 || a.max_seq_len <= 0 || a.position + a.n_steps > a.max_seq_len || a.max_seq_len > MAX_CTX) {
        set_error("position %d + %d steps exceeds max_seq_len %d (library limit %d)", a.position, a.n_steps, a.max_seq_len, MAX_CTX);
        return QWEN35_ERR_BAD_ARG;
    }
    if (!a.token_in && !a.forced_ids && (a.token_imm < 0 || a.token_imm >= VOCAB)) {
        set_error("token id %d out of range", a.token_imm);
        return QWEN35_ERR_BAD_ARG;
    }
    {
        const int g = decode_grid();
        if (g < 64 || g > 256) { set_error("needs between 64 and 256 SMs"); return QWEN35_ERR_UNSUPPORTED; }
        const int cap = (g / FA_KV_HEADS < ATT_MAX_CHUNKS ? g / FA_KV_HEADS : ATT_MAX_CHUNKS) * ATT_CHUNK_MAX;
        if (a.max_seq_len > cap) { set_error("max_seq_len %d exceeds %d on this device", a.max_seq_len, cap); return QWEN35_ERR_BAD_ARG; }
    }
    if (fp4 && !a.lm_scales) { set_error("NVFP4 decode needs the LM-head scales"); return QWEN35_ERR_BAD_ARG; }
    // The epoch counters and the static array's address are shared by every host thread that calls in on this
    // device: one lock covers the look-up, the epoch range hand-out and the launch, so ranges never overlap and
    // launches enter the stream in epoch order.
    static std::mutex launch_mu;
    std::lock_guard<std::mutex> lk(launch_mu);
    unsigned* epoch = use_static ? &g_static_epoch[dev] : &g_epoch[dev];
    if (use_static) {
        if (!g_static_ptr[dev]) {
            // once per device, with that device current: resolve the device address of the file-scope array
            void* p = nullptr;
            Q35_CUDA_OK(cudaGetSymbolAddress(&p, g_static_scratch));
            g_static_ptr[dev] = (StreamWorkspace*)p;
            register_status_word((int*)p);
        }
        a.ws = g_static_ptr[dev];
    } else {
        a.ws = (StreamWorkspace*)get_workspace();
    }
    if (!a.ws) return QWEN35_ERR_CUDA;
    // epochs tag every flagged word; they only ever grow, so words left by earlier calls never match.
    // On wrap-around the words are cleared (a memset, not an allocation).
    const unsigned long long need = 32ull * (unsigned long long)a.n_steps + 64ull;
    if ((unsigned long long)*epoch + need >= 0xffffff00ull) {
        Q35_CUDA_OK(cudaMemsetAsync((char*)a.ws + 256, 0, sizeof(StreamWorkspace) - 256, stream));
        *epoch = 0;
    }
    a.epoch_base = *epoch;
    a.tma_period = tma_period();
    void* params[] = {(void*)&a};
    const void* kern = fp4 ? (const void*)decode_stream_kernel<true> : (const void*)decode_stream_kernel<false>;
    Q35_CUDA_OK(cudaLaunchCooperativeKernel(kern, dim3(decode_grid()), dim3(STREAM_THREADS), params, sizeof(Smem), stream));
    *epoch += (unsigned)(32u * (unsigned)a.n_steps);      // only a launch that went out consumes its epoch range
    g_launches.fetch_add(1);
    return QWEN35_OK;
}

size_t workspace_bytes() { return sizeof(StreamWorkspace); }

}  // namespace q35

extern "C" int launch_decode(
    int input_token_id, int* output_token_id,
    const void* embed_weight, const LayerWeights* layer_weights,
    const void* final_norm_weight, const void* lm_head_weight,
    void* fa_k_cache, void* fa_v_cache, void* dn_states, void* conv_bufs,
    void* hidden_buffer, void*, void*, void*, void*, void*, void*, void*, void*, void*, void*,
    unsigned int*, unsigned int*, float*, int*, unsigned int*,
    int position, int max_seq_len, qwen35_stream_t stream) {
    q35::DecodeArgs a = {};
    a.layers = layer_weights;
    a.embed = (const q35::bf16*)embed_weight;
    a.final_norm = (const q35::bf16*)final_norm_weight;
    a.lm_head = (const q35::bf16*)lm_head_weight;
    a.k_cache = (q35::bf16*)fa_k_cache;
    a.v_cache = (q35::bf16*)fa_v_cache;
    a.dn_states = (float*)dn_states;
    a.conv_bufs = (float*)conv_bufs;
    a.token_imm = input_token_id;
    a.out_token = output_token_id;
    a.hidden_out = (q35::bf16*)hidden_buffer;
    a.position = position;
    a.max_seq_len = max_seq_len;
    a.n_steps = 1;
    return q35::launch_decode_impl(a, (cudaStream_t)stream);
}

static int decode_steps_common(const Qwen35DecodeArgs* in, qwen35_stream_t stream, bool use_static, bool fp4 = false, const void* lm_scales = nullptr) {
    if (!in) { q35::set_error("null args"); return QWEN35_ERR_BAD_ARG; }
    q35::DecodeArgs a = {};
    a.layers = in->layer_weights;
    a.embed = (const q35::bf16*)in->embed_weight;
    a.final_norm = (const q35::bf16*)in->final_norm_weight;
    a.lm_head = (const q35::bf16*)in->lm_head_weight;
    a.k_cache = (q35::bf16*)in->fa_k_cache;
    a.v_cache = (q35::bf16*)in->fa_v_cache;
    a.dn_states = (float*)in->dn_states;
    a.conv_bufs = (float*)in->conv_bufs;
    a.token_in = in->token_in;
    a.token_imm = in->token_imm;
    a.forced_ids = in->forced_ids;
    a.out_token = in->out_token;
    a.out_tokens = in->out_tokens;
    a.logits_out = in->logits_out;
    a.hidden_out = (q35::bf16*)in->hidden_out;
    a.dbg_hidden = (q35::bf16*)in->dbg_hidden;
    a.dbg_teacher = (const q35::bf16*)in->dbg_teacher;
    a.position = in->position;
    a.max_seq_len = in->max_seq_len;
    a.n_steps = in->n_steps;
    a.lm_last_only = in->lm_last_only;
    a.dbg_num_layers = in->dbg_num_layers;
    a.dbg_time = in->dbg_time;
    a.dbg_time_cta = in->dbg_time_cta;
    a.lm_scales = lm_scales;
    return q35::launch_decode_impl(a, (cudaStream_t)stream, use_static, fp4);
}

extern "C" int qwen35_b200_decode_steps(const Qwen35DecodeArgs* in, qwen35_stream_t stream) {
    return decode_steps_common(in, stream, false);
}

// Same kernel, same arguments, but the inter-stage scratch is the file-scope device array above instead of
// the workspace the library allocates on first use: this entry point never calls cudaMalloc, cudaFree or any
// other allocating routine.  Its first call on a device resolves the array's device address.
extern "C" int qwen35_b200_decode_steps_static(const Qwen35DecodeArgs* in, qwen35_stream_t stream) {
    if (in && in->max_seq_len > q35::MAX_CTX) {
        q35::set_error("max_seq_len %d exceeds the %d-token limit of the static scratch (%zu bytes)", in->max_seq_len, q35::MAX_CTX,
                       sizeof(q35::StreamWorkspace));
        return QWEN35_ERR_BAD_ARG;
    }
    return decode_steps_common(in, stream, true);
}

// ---- NVFP4 decode (reference: launch_decode_nvfp4 / launch_decode_many_nvfp4, kernel_gb10_nvfp4.cu:1999-2250) ----
static int nvfp4_common(const int* token_in, int* out_token, int* out_tokens, int steps,
                        const void* embed, const void* layers, const void* final_norm, const void* lm_packed, const void* lm_scales,
                        void* k_cache, void* v_cache, void* dn_states, void* conv_bufs, void* hidden, int position, int max_seq_len,
                        int group_size, qwen35_stream_t stream) {
    if (group_size != 32) { q35::set_error("NVFP4 decode supports group_size 32 (got %d)", group_size); return QWEN35_ERR_UNSUPPORTED; }
    if (!token_in) { q35::set_error("null token pointer"); return QWEN35_ERR_BAD_ARG; }
    q35::DecodeArgs a = {};
    a.layers = layers; a.embed = (const q35::bf16*)embed; a.final_norm = (const q35::bf16*)final_norm;
    a.lm_head = (const q35::bf16*)lm_packed; a.lm_scales = lm_scales;
    a.k_cache = (q35::bf16*)k_cache; a.v_cache = (q35::bf16*)v_cache; a.dn_states = (float*)dn_states; a.conv_bufs = (float*)conv_bufs;
    a.token_in = token_in; a.out_token = out_token; a.out_tokens = out_tokens; a.hidden_out = (q35::bf16*)hidden;
    a.position = position; a.max_seq_len = max_seq_len; a.n_steps = steps;
    return q35::launch_decode_impl(a, (cudaStream_t)stream, false, true);
}

extern "C" int launch_decode_nvfp4(
    const int* input_token_ptr, int* output_token_id, const void* embed_weight, const void* layer_weights,
    const void* final_norm_weight, const void* lm_head_weight_packed, const void* lm_head_scales,
    void*, void*, void*, void*,
    void* fa_k_cache, void* fa_v_cache, void* dn_states, void* conv_bufs, void* hidden_buffer,
    void*, void*, void*, void*, void*, void*, void*, void*, void*, void*,
    unsigned int*, unsigned int*, float*, int*, unsigned int*,
    int position, int max_seq_len, int group_size, qwen35_stream_t stream) {
    return nvfp4_common(input_token_ptr, output_token_id, nullptr, 1, embed_weight, layer_weights, final_norm_weight, lm_head_weight_packed,
                        lm_head_scales, fa_k_cache, fa_v_cache, dn_states, conv_bufs, hidden_buffer, position, max_seq_len, group_size, stream);
}

extern "C" int launch_decode_many_nvfp4(
    int* token_buffer, int* output_tokens, int steps, const void* embed_weight, const void* layer_weights,
    const void* final_norm_weight, const void* lm_head_weight_packed, const void* lm_head_scales,
    void*, void*, void*, void*,
    void* fa_k_cache, void* fa_v_cache, void* dn_states, void* conv_bufs, void* hidden_buffer,
    void*, void*, void*, void*, void*, void*, void*, void*, void*, void*,
    unsigned int*, unsigned int*, float*, int*, unsigned int*,
    int position, int max_seq_len, int group_size, qwen35_stream_t stream) {
    // token_buffer[0] holds the first input token and receives the last generated one, as in the reference
    return nvfp4_common(token_buffer, token_buffer, output_tokens, steps, embed_weight, layer_weights, final_norm_weight, lm_head_weight_packed,
                        lm_head_scales, fa_k_cache, fa_v_cache, dn_states, conv_bufs, hidden_buffer, position, max_seq_len, group_size, stream);
}

// Replaces launch_prefill_megakernel_nvfp4 (torch_bindings.cpp:104-119; prefill_kernel_nvfp4, kernel_gb10_nvfp4.cu:1659-1755,
// launcher :2119-2183): the prompt pass of the NVFP4 path, token-serial in the reference as well -- the decode megakernel is
// run over the seq_len prompt tokens from position 0 in one launch and the LM head only after the last one.
extern "C" int launch_prefill_megakernel_nvfp4(
    const int* token_ids, int seq_len, int* output_token_id, const void* embed_weight, const void* layer_weights,
    const void* final_norm_weight, const void* lm_head_weight_packed, const void* lm_head_scales,
    void*, void*, void*, void*,
    void* fa_k_cache, void* fa_v_cache, void* dn_states, void* conv_bufs, void* hidden_buffer,
    void*, void*, void*, void*, void*, void*, void*, void*, void*, void*,
    unsigned int*, unsigned int*, float*, int*, unsigned int*,
    int max_seq_len, int group_size, qwen35_stream_t stream) {
    if (group_size != 32) { q35::set_error("NVFP4 decode supports group_size 32 (got %d)", group_size); return QWEN35_ERR_UNSUPPORTED; }
    if (!token_ids || seq_len <= 0) { q35::set_error("prefill_megakernel_nvfp4: no prompt tokens"); return QWEN35_ERR_BAD_ARG; }
    q35::DecodeArgs a = {};
    a.layers = layer_weights; a.embed = (const q35::bf16*)embed_weight; a.final_norm = (const q35::bf16*)final_norm_weight;
    a.lm_head = (const q35::bf16*)lm_head_weight_packed; a.lm_scales = lm_head_scales;
    a.k_cache = (q35::bf16*)fa_k_cache; a.v_cache = (q35::bf16*)fa_v_cache; a.dn_states = (float*)dn_states; a.conv_bufs = (float*)conv_bufs;
    a.forced_ids = token_ids; a.out_token = output_token_id; a.hidden_out = (q35::bf16*)hidden_buffer;
    a.position = 0; a.max_seq_len = max_seq_len; a.n_steps = seq_len; a.lm_last_only = 1;
    return q35::launch_decode_impl(a, (cudaStream_t)stream, false, true);
}

// Extended NVFP4 decode: the arguments of qwen35_b200_decode_steps (layer table in the NVFP4 record layout,
// lm_head_weight = packed nibbles) plus the LM-head scales.
extern "C" int qwen35_b200_decode_steps_nvfp4(const Qwen35DecodeArgs* in, const void* lm_head_scales, qwen35_stream_t stream) {
    return decode_steps_common(in, stream, false, true, lm_head_scales);
}

// Debug: synchronise the device and decode one flagged-word vector of the workspace to bf16 on the host.
// which: 0 = xa (8224), 1 = o (2048), 2 = h1 (1024), 3 = m (3584), 4 = h2 (1024)
extern "C" int qwen35_b200_debug_read(int which, void* host_out) {
    using namespace q35;
    StreamWorkspace* ws = (StreamWorkspace*)get_workspace();
    if (!ws || !host_out) return QWEN35_ERR_BAD_ARG;
    const u64* src; int n;
    switch (which) {
        case 0: src = ws->xa; n = DN_PROJ_ROWS / 2; break;
        case 1: src = ws->o; n = DN_V_SIZE / 2; break;
        case 2: src = ws->h1; n = HIDDEN / 2; break;
        case 3: src = ws->m; n = INTER / 2; break;
        case 4: src = ws->h2; n = HIDDEN / 2; break;
        default: return QWEN35_ERR_BAD_ARG;
    }
    static u64 tmp[DN_PROJ_ROWS / 2];
    Q35_CUDA_OK(cudaDeviceSynchronize());
    Q35_CUDA_OK(cudaMemcpy(tmp, src, (size_t)n * 8, cudaMemcpyDeviceToHost));
    for (int i = 0; i < n; ++i) ((uint32_t*)host_out)[i] = (uint32_t)tmp[i];
    return QWEN35_OK;
}

extern "C" int qwen35_b200_rope_inv_freq(float* host_out32) {
    if (!host_out32) return QWEN35_ERR_BAD_ARG;
    q35::rope_table(host_out32);
    return QWEN35_OK;
}
