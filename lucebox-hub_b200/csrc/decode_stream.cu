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

struct Smem {
    // ring first: 16-byte aligned slots
    unsigned char ring[NSLOTS * SLOT_BYTES];
    unsigned long long full[NSLOTS];
    unsigned long long empty[NSLOTS];
    LayerW layers[NUM_LAYERS];
    __align__(16) bf16 x[INTER];                 // GEMV input of the current stage
    __align__(16) bf16 h[HIDDEN];                // raw layer input (residual of stage C)
    __align__(16) bf16 h1[HIDDEN];               // raw mixer output (residual of stage E)
    float part[512];                             // cross-warp partial sums; attention chunk statistics
    float red[NCONS_WARPS];
    uint32_t stage[64];                          // packed outputs of a stage, published by one coalesced store
    __align__(16) float qk[2][2][DN_K];
    float hd[2][2];
    __align__(16) float q[FA_GQA][FA_HEAD_DIM];
    __align__(16) float kcur[FA_HEAD_DIM];
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
        if (a.dbg_time && last_step && tid == 0) a.dbg_time[((size_t)b * 25 + stamp_row) * 12 + (k)] = gtime(); \
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
    const int b = blockIdx.x, G = gridDim.x;
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
                for (int u = part_begin(TILES_A_DN, b, G); u < part_begin(TILES_A_DN, b + 1, G); ++u) {
                    const int v = u * 8;
                    if (v < DN_CONV_CH) issue_rows(L.p[W_A0], L.p[W_A0S], v, 8, HIDDEN);
                    else if (v < DN_CONV_CH + DN_V_SIZE) issue_rows(L.p[W_A1], L.p[W_A1S], v - DN_CONV_CH, 8, HIDDEN);
                    else if (v < DN_CONV_CH + DN_V_SIZE + DN_HEADS) issue_rows(L.p[W_A2], nullptr, v - DN_CONV_CH - DN_V_SIZE, 8, HIDDEN);
                    else issue_rows(L.p[W_A3], nullptr, v - DN_CONV_CH - DN_V_SIZE - DN_HEADS, 8, HIDDEN);
                }
            } else {
                for (int u = part_begin(TILES_A_FA, b, G); u < part_begin(TILES_A_FA, b + 1, G); ++u) {
                    const int v = u * 8;
                    if (v < FA_QPROJ) issue_rows(L.p[W_A0], L.p[W_A0S], v, 8, HIDDEN);
                    else if (v < FA_QPROJ + FA_KV_SIZE) issue_rows(L.p[W_A1], L.p[W_A1S], v - FA_QPROJ, 8, HIDDEN);
                    else issue_rows(L.p[W_A2], L.p[W_A2S], v - FA_QPROJ - FA_KV_SIZE, 8, HIDDEN);
                }
            }
            for (int u = part_begin(TILES_C, b, G); u < part_begin(TILES_C, b + 1, G); ++u) issue_rows(L.p[W_OUT], L.p[W_OUTS], u * 4, 4, 2048);
            for (int u = part_begin(UNITS_D, b, G); u < part_begin(UNITS_D, b + 1, G); ++u) {
                issue_rows(L.p[W_GATE], L.p[W_GATES], u * 8, 8, HIDDEN);
                issue_rows(L.p[W_UP], L.p[W_UPS], u * 8, 8, HIDDEN);
            }
            for (int u = part_begin(TILES_E, b, G); u < part_begin(TILES_E, b + 1, G); ++u) issue_rows(L.p[W_DOWN], L.p[W_DOWNS], u * 2, 2, INTER);
        }
        if (!a.lm_last_only || step == a.n_steps - 1) {
            if (!FP4) {
                for (int u = part_begin(TILES_LM, b, G); u < part_begin(TILES_LM, b + 1, G); ++u)
                    issue((const char*)a.lm_head + (size_t)u * SLOT_BYTES, SLOT_BYTES, nullptr, 0);
            } else {
                // per 128-row block: its 8 KB of swizzled E4M3 scales, then four 32-row tiles of packed nibbles
                for (int blk = part_begin(FP4_LM_BLOCKS, b, G); blk < part_begin(FP4_LM_BLOCKS, b + 1, G); ++blk) {
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
// NMAT = 2 pairs a gate tile with an up tile.  epi(first_row_of_pair, sums[NMAT][2]) runs on lane 0.
template <int NMAT, typename Epi>
__device__ __forceinline__ void consume_k1024(Ring& ring, int n_units, const bf16* xs, const Abort& ab, Epi epi) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float x[32];
#pragma unroll
    for (int j = 0; j < 4; ++j) unpack8(*reinterpret_cast<const uint4*>(xs + (j * 32 + lane) * 8), x + 8 * j);
    const unsigned t0 = ring.t;
    for (int g = 0; g < n_units; g += 4) {
        const int ui = g + (warp >> 2);
        if (ui < n_units) {
            float acc[NMAT][2];
#pragma unroll
            for (int m = 0; m < NMAT; ++m) {
                const unsigned tile = t0 + (unsigned)(ui * NMAT + m);
                mbar_wait(ring.full_bar(tile), ring.phase(tile), ab);
                const uint32_t base = ring.slot_addr(tile) + (uint32_t)(2 * (warp & 3)) * 2048u + (uint32_t)lane * 16u;
                uint4 w0[4], w1[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) { w0[j] = lds128(base + j * 512); w1[j] = lds128(base + 2048 + j * 512); }
                float a0 = 0.f, a1 = 0.f;
#pragma unroll
                for (int j = 0; j < 4; ++j) { a0 = dot8(w0[j], x + 8 * j, a0); a1 = dot8(w1[j], x + 8 * j, a1); }
                acc[m][0] = warp_sum(a0);
                acc[m][1] = warp_sum(a1);
                if (lane == 0) mbar_arrive(ring.empty_bar(tile), 4);
            }
            if (lane == 0) epi(ui * 8 + 2 * (warp & 3), acc);
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
__device__ __forceinline__ void consume_k1024_fp4(Ring& ring, int n_units, const bf16* xs, const Abort& ab, Epi epi) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float x[32];
    load_x32(xs, 32 * lane, x);
    const unsigned t0 = ring.t;
    for (int g = 0; g < n_units; g += 4) {
        const int ui = g + (warp >> 2);
        if (ui < n_units) {
            float acc[NMAT][2];
#pragma unroll
            for (int m = 0; m < NMAT; ++m) {
                const unsigned tile = t0 + (unsigned)(ui * NMAT + m);
                mbar_wait(ring.full_bar(tile), ring.phase(tile), ab);
                const uint32_t r0 = (uint32_t)(2 * (warp & 3));
                const uint32_t base = ring.slot_addr(tile) + r0 * 512u + (uint32_t)lane * 16u;
                const uint32_t sbase = ring.slot_addr(tile) + FP4_SCALE_OFF + r0 * 64u + (uint32_t)lane * 2u;
                const uint4 p0 = lds128(base), p1 = lds128(base + 512);
                const float s0 = lds_half(sbase), s1 = lds_half(sbase + 64);
                acc[m][0] = warp_sum(dot32_fp4(p0, x) * s0);
                acc[m][1] = warp_sum(dot32_fp4(p1, x) * s1);
                if (lane == 0) mbar_arrive(ring.empty_bar(tile), 4);
            }
            if (lane == 0) epi(ui * 8 + 2 * (warp & 3), acc);
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

// RMSNorm(1+w) of 1024 values held one pair per consumer thread; writes bf16 to xs.
__device__ __forceinline__ void rmsnorm_pair(uint32_t raw, const bf16* w, bf16* xs, float* s_red) {
    const int t = threadIdx.x;
    const float x0 = bf_lo(raw), x1 = bf_hi(raw);
    const float tot = cons_block_sum(x0 * x0 + x1 * x1, s_red);
    const float r = rsqrt_ieee(tot * (1.0f / HIDDEN) + RMS_EPS);
    const uint32_t wr = __ldg(reinterpret_cast<const uint32_t*>(w) + t);
    reinterpret_cast<uint32_t*>(xs)[t] = pack_bf16x2((x0 * r) * (1.0f + bf_lo(wr)), (x1 * r) * (1.0f + bf_hi(wr)));
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
        mbar_fence_init();
    }
    if (tid < NUM_LAYERS) load_layer<FP4>(a.layers, tid, s.layers[tid]);
    __syncthreads();

    Abort ab{&s.abort_flag, &ws->err};
    Ring ring{smem_u32(s.ring), smem_u32(s.full), smem_u32(s.empty), 0u};

    if (warp == NCONS_WARPS) {
        if (lane == 0) produce<FP4>(a, s, ring, ab);
        __syncwarp();
    } else {
        // =========================== consumers ===========================
        int tok = a.token_in ? __ldg(a.token_in) : a.token_imm;
        const int n_layers = a.dbg_num_layers > 0 ? a.dbg_num_layers : NUM_LAYERS;
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
                const bf16* w_post = (const bf16*)L.p[W_POST_NORM];

                // ---- DeltaNet: issue the state / conv loads of stage B before any waiting ----
                const int pp0 = part_begin(DN_V_SIZE / 2, b, G), pp1 = part_begin(DN_V_SIZE / 2, b + 1, G);   // value-row pairs
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
                    uint32_t raw;
                    if (layer == 0) raw = __ldg(reinterpret_cast<const uint32_t*>(a.embed + (size_t)tok * HIDDEN) + tid);
                    else if (a.dbg_teacher) raw = __ldg(reinterpret_cast<const uint32_t*>(a.dbg_teacher + layer * HIDDEN) + tid);
                    else raw = poll_word(&ws->h2[tid], epoch_of(a, step, layer - 1), ab);
                    reinterpret_cast<uint32_t*>(s.h)[tid] = raw;
                    rmsnorm_pair(raw, (const bf16*)L.p[W_IN_NORM], s.x, s.red);
                    cons_sync();
                    Q35_STAMP(1);
                    const int ntl = dn ? TILES_A_DN : TILES_A_FA;
                    const int u0 = part_begin(ntl, b, G), u1 = part_begin(ntl, b + 1, G);
                    if (FP4) {
                        // qkv / z (or q, k, v) tiles are NVFP4; the 16+16 rows of the b and a projections stay bf16
                        const int n_q = dn ? max(0, min(u1, (DN_CONV_CH + DN_V_SIZE) / 8) - u0) : (u1 - u0);
                        consume_k1024_fp4<1>(ring, n_q, s.x, ab, [&](int row, const float (*acc)[2]) {
                            s.stage[row >> 1] = pack_bf16x2(acc[0][0], acc[0][1]);
                        });
                        if (u1 - u0 > n_q)
                            consume_k1024<1>(ring, u1 - u0 - n_q, s.x, ab, [&](int row, const float (*acc)[2]) {
                                s.stage[(n_q * 8 + row) >> 1] = pack_bf16x2(acc[0][0], acc[0][1]);
                            });
                    } else {
                        consume_k1024<1>(ring, u1 - u0, s.x, ab, [&](int row, const float (*acc)[2]) {
                            s.stage[row >> 1] = pack_bf16x2(acc[0][0], acc[0][1]);
                        });
                    }
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
                        if (lane == 0) s.stage[warp] = pack_bf16x2(ov[0], ov[1]);
                    }
                    cons_sync();
                    if (tid < pp1 - pp0) st_word(&ws->o[pp0 + tid], s.stage[tid], ep);

                    Q35_STAMP(3);
                    // ================= stage C (DeltaNet): gated norm (one head per warp), conv shift =================
                    {
                        const int h = warp;
                        uint32_t o0, o1, z0, z1;
                        {
                            // z was published in stage A, long ago: its loads overlap the wait for `o`
                            const u64* po = &ws->o[h * 64 + lane * 2];
                            const u64* pz = &ws->xa[(DN_CONV_CH >> 1) + h * 64 + lane * 2];
                            const u64 b0 = ld_word(pz), b1 = ld_word(pz + 1);
                            poll2(po, po + 1, ep, ab, o0, o1);
                            z0 = ((uint32_t)(b0 >> 32) == ep) ? (uint32_t)b0 : poll_word(pz, ep, ab);
                            z1 = ((uint32_t)(b1 >> 32) == ep) ? (uint32_t)b1 : poll_word(pz + 1, ep, ab);
                        }
                        const uint2 nrw = __ldg(reinterpret_cast<const uint2*>(L.p[W_GNORM]) + lane);
                        const float ov[4] = {bf_lo(o0), bf_hi(o0), bf_lo(o1), bf_hi(o1)};
                        const float zv[4] = {bf_lo(z0), bf_hi(z0), bf_lo(z1), bf_hi(z1)};
                        const float nw[4] = {bf_lo(nrw.x), bf_hi(nrw.x), bf_lo(nrw.y), bf_hi(nrw.y)};
                        const float var = warp_sum(ov[0] * ov[0] + ov[1] * ov[1] + ov[2] * ov[2] + ov[3] * ov[3]) * (1.0f / DN_V);
                        const float r = rsqrt_ieee(var + RMS_EPS);
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            const float n = rbf(ov[i] * r);
                            const float t = rbf(nw[i] * n);
                            s.x[h * DN_V + lane * 4 + i] = f2bf(t * silu_f(zv[i]));
                        }
                    }
                    ++i_dn;
                } else {
                    // ================= attention: B1 scores + chunk statistics, B2 P.V partials, B3 merge + gate =================
                    // The context is split into chunks of >= 32 positions; CTA (kv head, chunk) owns one chunk.
                    bf16* kc = a.k_cache + (size_t)i_fa * FA_KV_HEADS * a.max_seq_len * FA_HEAD_DIM;
                    bf16* vc = a.v_cache + (size_t)i_fa * FA_KV_HEADS * a.max_seq_len * FA_HEAD_DIM;
                    const int Lc = pos + 1;
                    int nchunk = (Lc + 31) / 32;
                    { const int cap = min(ATT_MAX_CHUNKS, G / FA_KV_HEADS); if (nchunk > cap) nchunk = cap; }
                    const int clen = (Lc + nchunk - 1) / nchunk;            // <= ATT_CHUNK_MAX by the host-side limit on max_seq_len
                    const bool att_cta = b < FA_KV_HEADS * nchunk;
                    const int kvh = b / nchunk, chunk = b % nchunk;
                    const int j0 = chunk * clen, j1 = min(Lc, j0 + clen);
                    if (att_cta) {
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
                            if (!isq && pos >= j0 && pos < j1) {
                                uint32_t* krow = reinterpret_cast<uint32_t*>(kc + ((size_t)kvh * a.max_seq_len + pos) * FA_HEAD_DIM);
#pragma unroll
                                for (int i = 0; i < 4; ++i) krow[lane + 32 * i] = pack_bf16x2(xv[2 * i], xv[2 * i + 1]);
                                __threadfence();
                            }
                        } else if (warp == FA_GQA + 1 && pos >= j0 && pos < j1) {
                            uint32_t* vrow = reinterpret_cast<uint32_t*>(vc + ((size_t)kvh * a.max_seq_len + pos) * FA_HEAD_DIM);
                            uint32_t wv[4];
                            poll4(&ws->xa[((FA_QPROJ + FA_KV_SIZE + kvh * FA_HEAD_DIM) >> 1) + lane], 32, ep, ab, wv);
#pragma unroll
                            for (int i = 0; i < 4; ++i) vrow[lane + 32 * i] = wv[i];
                            __threadfence();
                        }
                        cons_sync();
                        // ---- scores of this chunk, two positions per warp in flight ----
                        {
                            float qr[FA_GQA][8];
#pragma unroll
                            for (int g = 0; g < FA_GQA; ++g)
#pragma unroll
                                for (int i = 0; i < 8; ++i) qr[g][i] = s.q[g][lane * 8 + i];
                            for (int j = j0 + warp; j < j1; j += 2 * NCONS_WARPS) {
                                const int jb = j + NCONS_WARPS;
                                uint4 ka = make_uint4(0, 0, 0, 0), kb = ka;
                                if (j != pos) ka = ld_cg(reinterpret_cast<const uint4*>(kc + ((size_t)kvh * a.max_seq_len + j) * FA_HEAD_DIM) + lane);
                                if (jb < j1 && jb != pos) kb = ld_cg(reinterpret_cast<const uint4*>(kc + ((size_t)kvh * a.max_seq_len + jb) * FA_HEAD_DIM) + lane);
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
                                for (int u = 0; u < 32; ++u) vr[u] = (jj + u < cn) ? ld_cg(vb + (size_t)(jj + u) * (FA_HEAD_DIM / 2)) : 0u;
#pragma unroll
                                for (int u = 0; u < 32; ++u) {
                                    const float p = (jj + u < cn) ? s.p[g][jj + u] : 0.f;
                                    acc0 = fmaf(p, bf_lo(vr[u]), acc0);
                                    acc1 = fmaf(p, bf_hi(vr[u]), acc1);
                                }
                            }
                            reinterpret_cast<float2*>(ws->att_part[chunk][kvh * FA_GQA + g])[d2] = make_float2(acc0, acc1);
                        }
                        __threadfence();
                        cons_sync();
                        if (tid == 0) st_release(&ws->att_flag[kvh][chunk], ep);
                    }
                    // ---- B3: CTA h < 8 merges the partials of query head h and applies the sigmoid gate ----
                    if (b < FA_Q_HEADS) {
                        const int qh = b;
                        if (tid < nchunk) {
                            unsigned it = 0;
                            while (ld_acquire(&ws->att_flag[qh / FA_GQA][tid]) != ep && !ab.on()) {
                                if (++it > POLL_LIMIT) { ab.raise(ERR_BARRIER_TIMEOUT); break; }
                            }
                        }
                        cons_sync();
                        {
                            // 8 groups of 64 threads: group q sums chunks q, q+8, ... (all its loads in flight at once: one L2
                            // round trip), then thread t < 64 adds the 8 group sums in group order and applies the gate
                            const int d = (tid & 63) * 4, grp = tid >> 6;
                            float4 pv[ATT_MAX_CHUNKS / 8];
#pragma unroll
                            for (int u = 0; u < ATT_MAX_CHUNKS / 8; ++u) {
                                const int c = grp + 8 * u;
                                pv[u] = (c < nchunk) ? ld_cg(reinterpret_cast<const float4*>(&ws->att_part[c][qh][d])) : make_float4(0.f, 0.f, 0.f, 0.f);
                            }
                            float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
                            for (int u = 0; u < ATT_MAX_CHUNKS / 8; ++u) { acc.x += pv[u].x; acc.y += pv[u].y; acc.z += pv[u].z; acc.w += pv[u].w; }
                            reinterpret_cast<float4*>(&s.p[0][0])[tid] = acc;         // P of this CTA's chunk is no longer needed: [8 groups][64 x float4]
                        }
                        cons_sync();
                        if (tid < 64) {
                            const int d = tid * 4;
                            uint32_t g0, g1;
                            const int ge = qh * 2 * FA_HEAD_DIM + FA_HEAD_DIM + d;
                            poll2(&ws->xa[ge >> 1], &ws->xa[(ge >> 1) + 1], ep, ab, g0, g1);
                            float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
                            for (int q = 0; q < 8; ++q) {
                                const float4 v = reinterpret_cast<const float4*>(&s.p[0][0])[q * 64 + tid];
                                acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
                            }
                            const float u0 = rbf(acc.x) * rbf(sigmoid_f(bf_lo(g0))), u1 = rbf(acc.y) * rbf(sigmoid_f(bf_hi(g0)));
                            const float u2 = rbf(acc.z) * rbf(sigmoid_f(bf_lo(g1))), u3 = rbf(acc.w) * rbf(sigmoid_f(bf_hi(g1)));
                            st_word(&ws->o[(qh * FA_HEAD_DIM + d) >> 1], pack_bf16x2(u0, u1), ep);
                            st_word(&ws->o[((qh * FA_HEAD_DIM + d) >> 1) + 1], pack_bf16x2(u2, u3), ep);
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
                Q35_STAMP(4);
                // ---- stage C tail: output projection (K = 2048, 4 rows per tile) + residual ----
                {
                    const bf16* hin = s.h;
                    const int u0 = part_begin(TILES_C, b, G), nt = part_begin(TILES_C, b + 1, G) - u0;
                    if (FP4) {
                        // 4 rows x 1024 bytes of nibbles per tile; warps 0-7: row w/2, K half w%2 (32 groups of 32, one per lane)
                        float x[32];
                        if (warp < 8) load_x32(s.x, (warp & 1) * 1024 + 32 * lane, x);
                        for (int ti = 0; ti < nt; ++ti) {
                            const unsigned tile = ring.t + (unsigned)ti;
                            if (warp < 8) {
                                mbar_wait(ring.full_bar(tile), ring.phase(tile), ab);
                                const uint32_t row = (uint32_t)(warp >> 1), half = (uint32_t)(warp & 1);
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
                    float x[16];
                    unpack8(*reinterpret_cast<const uint4*>(s.x + (warp & 3) * 512 + lane * 8), x);
                    unpack8(*reinterpret_cast<const uint4*>(s.x + (warp & 3) * 512 + (32 + lane) * 8), x + 8);
                    for (int ti = 0; ti < nt; ++ti) {
                        const unsigned tile = ring.t + (unsigned)ti;
                        mbar_wait(ring.full_bar(tile), ring.phase(tile), ab);
                        const uint32_t base = ring.slot_addr(tile) + (uint32_t)(warp >> 2) * 4096u + (uint32_t)(warp & 3) * 1024u + (uint32_t)lane * 16u;
                        const uint4 q0 = lds128(base), q1 = lds128(base + 512);
                        const float acc = warp_sum(dot8(q1, x + 8, dot8(q0, x, 0.f)));
                        if (lane == 0) { s.part[ti * 16 + warp] = acc; mbar_arrive(ring.empty_bar(tile), 1); }
                    }
                    }
                    ring.t += (unsigned)nt;
                    cons_sync();
                    if (tid < nt * 2) {
                        const int ti = tid >> 1, pr = tid & 1;
                        const float* pp = &s.part[ti * 16 + pr * 8];
                        const float y0 = ((pp[0] + pp[1]) + pp[2]) + pp[3], y1 = ((pp[4] + pp[5]) + pp[6]) + pp[7];
                        const int row = (u0 + ti) * 4 + 2 * pr;
                        st_word(&ws->h1[row >> 1], pack_bf16x2(bf2f(hin[row]) + rbf(y0), bf2f(hin[row + 1]) + rbf(y1)), ep);
                    }
                }

                Q35_STAMP_ALL(5);
                if (dn) {
                    // Conv-window shift, off the critical path.  This CTA has seen all of `o`, so every CTA
                    // finished stage B and nobody reads this layer's old window any more.  The fence orders the
                    // new window before this CTA's next publication (stage D), which the next token's readers follow.
                    for (int c = part_begin(DN_CONV_CH / 2, b, G) + tid; c < part_begin(DN_CONV_CH / 2, b + 1, G); c += NCONS) {
                        const uint32_t xw = poll_word(&ws->xa[c], ep, ab);
                        const float4 c0 = ld_cg(reinterpret_cast<const float4*>(conv) + 2 * c);
                        const float4 c1 = ld_cg(reinterpret_cast<const float4*>(conv) + 2 * c + 1);
                        reinterpret_cast<float4*>(conv)[2 * c] = make_float4(c0.y, c0.z, c0.w, bf_lo(xw));
                        reinterpret_cast<float4*>(conv)[2 * c + 1] = make_float4(c1.y, c1.z, c1.w, bf_hi(xw));
                        __threadfence();
                    }
                }
                // ================= stage D: post norm, gate/up with SiLU*up =================
                {
                    const uint32_t raw = poll_word(&ws->h1[tid], ep, ab);
                    reinterpret_cast<uint32_t*>(s.h1)[tid] = raw;
                    rmsnorm_pair(raw, w_post, s.x, s.red);
                    cons_sync();
                    Q35_STAMP(6);
                    const int u0 = part_begin(UNITS_D, b, G), u1 = part_begin(UNITS_D, b + 1, G);
                    auto epi_d = [&](int row, const float (*acc)[2]) {
                        const float m0 = rbf(silu_f(rbf(acc[0][0]))) * rbf(acc[1][0]);
                        const float m1 = rbf(silu_f(rbf(acc[0][1]))) * rbf(acc[1][1]);
                        s.stage[row >> 1] = pack_bf16x2(m0, m1);
                    };
                    if (FP4) consume_k1024_fp4<2>(ring, u1 - u0, s.x, ab, epi_d);
                    else consume_k1024<2>(ring, u1 - u0, s.x, ab, epi_d);
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
                    const int u0 = part_begin(TILES_E, b, G), nt = part_begin(TILES_E, b + 1, G) - u0;
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
                            float acc = 0.f;
#pragma unroll
                            for (int j = 0; j < 7; ++j) acc = dot8p(lds128(base + j * 512), xp[j], acc);
                            acc = warp_sum(acc);
                            if (lane == 0) { s.part[ti * 4 + (warp & 3)] = acc; mbar_arrive(ring.empty_bar(tile), 4); }
                        }
                    }
                    }
                    ring.t += (unsigned)nt;
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
                const uint32_t raw = poll_word(&ws->h2[tid], epoch_of(a, step, n_layers - 1), ab);
                Q35_STAMP(1);
                rmsnorm_pair(raw, a.final_norm, s.x, s.red);
                cons_sync();
                float best = -INFINITY;
                int best_i = 0x7fffffff;
                float* lg = (last_step ? a.logits_out : nullptr);
                // rows of the vocabulary owned by this CTA: [lm_row0, ...), in 8-row tiles (bf16) or 128-row blocks (NVFP4)
                const int lm_row0 = FP4 ? part_begin(FP4_LM_BLOCKS, b, G) * 128 : part_begin(TILES_LM, b, G) * 8;
                if (FP4) {
                    // tensor-core layout: one E4M3 scale per 16 weights, stored in 512-byte tiles of 128 rows x 4 blocks
                    float x[32];
                    load_x32(s.x, 32 * lane, x);
                    const int B0 = part_begin(FP4_LM_BLOCKS, b, G), B1 = part_begin(FP4_LM_BLOCKS, b + 1, G);
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
                    const int u0 = part_begin(TILES_LM, b, G), u1 = part_begin(TILES_LM, b + 1, G);
                    consume_k1024<1>(ring, u1 - u0, s.x, ab, [&](int row, const float (*acc)[2]) {
                        const int r0 = u0 * 8 + row;
                        const float v0 = rbf(acc[0][0]), v1 = rbf(acc[0][1]);
                        if (lg) { lg[r0] = v0; lg[r0 + 1] = v1; }
                        if (v0 > best) { best = v0; best_i = r0; }
                        if (v1 > best) { best = v1; best_i = r0 + 1; }
                    });
                }
                Q35_STAMP(2);
                // lane 0 of every warp holds that warp's best (rows ascend within a warp)
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
                            const int idx = (FP4 ? part_begin(FP4_LM_BLOCKS, c, G) * 128 : part_begin(TILES_LM, c, G) * 8) + (int)(w & 0xffffu);
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
