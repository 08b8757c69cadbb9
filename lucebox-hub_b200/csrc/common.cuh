// Shared device helpers for the Qwen3.5-0.8B hybrid forward kernels (sm_100a).
//
// Model constants restate models/qwen35_0p8b/kernel.cu:23-49 of the reference; the layer
// record mirrors `struct LayerWeights` (kernel.cu:77-115): int type, 3 pad ints, 14 pointers.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace q35 {

constexpr int HIDDEN = 1024;
constexpr int INTER = 3584;
constexpr int NUM_LAYERS = 24;
constexpr int VOCAB = 248320;
constexpr float RMS_EPS = 1e-6f;

constexpr int FA_Q_HEADS = 8;
constexpr int FA_KV_HEADS = 2;
constexpr int FA_GQA = FA_Q_HEADS / FA_KV_HEADS;
constexpr int FA_HEAD_DIM = 256;
constexpr int FA_Q_SIZE = FA_Q_HEADS * FA_HEAD_DIM;        // 2048
constexpr int FA_QPROJ = 2 * FA_Q_SIZE;                    // 4096: per head [q(256) | gate(256)]
constexpr int FA_KV_SIZE = FA_KV_HEADS * FA_HEAD_DIM;      // 512
constexpr int FA_PROJ_ROWS = FA_QPROJ + 2 * FA_KV_SIZE;    // 5120
constexpr int FA_ROT = 64;
constexpr int N_FA = 6;

constexpr int DN_HEADS = 16;
constexpr int DN_K = 128;
constexpr int DN_V = 128;
constexpr int DN_QK_SIZE = DN_HEADS * DN_K;                // 2048
constexpr int DN_V_SIZE = DN_HEADS * DN_V;                 // 2048
constexpr int DN_CONV_CH = 2 * DN_QK_SIZE + DN_V_SIZE;     // 6144
constexpr int DN_PROJ_ROWS = DN_CONV_CH + DN_V_SIZE + 2 * DN_HEADS;  // 8224: qkv | z | b | a
constexpr int N_DN = 18;

constexpr int NTHREADS = 512;
constexpr int NWARPS = NTHREADS / 32;

struct LayerRec {
    int type;            // 0 = DeltaNet, 1 = full attention
    int pad[3];
    const void* p[14];
};
static_assert(sizeof(LayerRec) == 128, "layer record is 128 bytes");

// Fused prefill weights of one layer (reference: struct PrefillFusedLayerWeights, torch_bindings.cpp:31-38, prefill.cu:66-73).
struct PrefillFused {
    const void* proj_weight;     // DN: [qkv; z; b; a] = 8224 x 1024, FA: [q; k; v] = 5120 x 1024
    const void* gate_up_weight;  // [gate; up] = 7168 x 1024
    const void* proj_packed;     // optional NVFP4 (tensor-core layout) copies of the same two matrices: packed nibbles and scale atoms;
    const void* proj_scales;     // DeltaNet projection rows padded to 8320.  When all four are set (and the caller did not switch it
    const void* gate_up_packed;  // off) the two GEMMs run block-scaled on FP4 operands, activations quantised on the way
    const void* gate_up_scales;  // (reference: prefill.cu:1210-1262, 1330-1347)
};
// Host copies of the two device tables, cached per pair of device addresses by the prefill launcher.
struct HostTables { const void* dev_layers; const void* dev_fused; LayerRec layers[NUM_LAYERS]; PrefillFused fused[NUM_LAYERS]; };
bool host_layer_tables(const void* dev_layers, const void* dev_fused, HostTables* out);

// Pointer slots (models/qwen35_0p8b/model.py:342-380).
enum FaSlot { FA_IN_NORM = 0, FA_Q, FA_K, FA_V, FA_QNORM, FA_KNORM, FA_O, FA_POST_NORM, FA_GATE, FA_UP, FA_DOWN };
enum DnSlot { DN_IN_NORM = 0, DN_QKV, DN_Z, DN_B, DN_A, DN_CONV, DN_ALOG, DN_DTBIAS, DN_NORM, DN_OUT, DN_POST_NORM,
              DN_GATE, DN_UP, DN_DOWN };

typedef __nv_bfloat16 bf16;

// ---- scalar helpers -----------------------------------------------------------------------
__device__ __forceinline__ float bf_lo(uint32_t u) { return __uint_as_float(u << 16); }
__device__ __forceinline__ float bf_hi(uint32_t u) { return __uint_as_float(u & 0xffff0000u); }
__device__ __forceinline__ float bf2f(bf16 v) { return __bfloat162float(v); }
__device__ __forceinline__ bf16 f2bf(float v) { return __float2bfloat16_rn(v); }
// round to bf16 and widen again: the value an op that returns bf16 hands to the next op
__device__ __forceinline__ float rbf(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

__device__ __forceinline__ float sigmoid_f(float x) { return 1.0f / (1.0f + expf(-x)); }
__device__ __forceinline__ float silu_f(float x) { return x / (1.0f + expf(-x)); }
__device__ __forceinline__ float rsqrt_ieee(float x) { return 1.0f / sqrtf(x); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// ---- memory helpers -----------------------------------------------------------------------
// Weights: read once per token, never written by a kernel -> non-coherent path, no L1 allocation.
__device__ __forceinline__ uint4 ld_stream(const uint4* p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
    return r;
}
// Activations written by other CTAs earlier in the same launch: L2-coherent loads.
__device__ __forceinline__ uint4 ld_cg(const uint4* p) { return __ldcg(p); }
__device__ __forceinline__ uint2 ld_cg(const uint2* p) { return __ldcg(p); }
__device__ __forceinline__ uint32_t ld_cg(const uint32_t* p) { return __ldcg(p); }
__device__ __forceinline__ float ld_cg(const float* p) { return __ldcg(p); }
__device__ __forceinline__ float4 ld_cg(const float4* p) { return __ldcg(p); }
__device__ __forceinline__ float ld_cg_bf16(const bf16* p) {
    return bf2f(__ushort_as_bfloat16(__ldcg(reinterpret_cast<const unsigned short*>(p))));
}

__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release(unsigned* p, unsigned v) {
    asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int ld_volatile(const int* p) {
    int v;
    asm volatile("ld.volatile.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// [b*n/G, (b+1)*n/G): contiguous, balanced to within one unit.
__device__ __forceinline__ int part_begin(int n, int b, int G) { return (int)(((long long)n * b) / G); }

// ---- block reductions ---------------------------------------------------------------------
// Sum over the CTA; every thread gets the result.  `scratch` holds NWARPS floats.
__device__ __forceinline__ float block_sum(float v, float* scratch) {
    v = warp_sum(v);
    __syncthreads();
    if ((threadIdx.x & 31) == 0) scratch[threadIdx.x >> 5] = v;
    __syncthreads();
    float t = 0.f;
#pragma unroll
    for (int i = 0; i < NWARPS; ++i) t += scratch[i];
    return t;
}

// ---- grid barrier with a bounded wait -----------------------------------------------------
// All CTAs of a cooperative launch are co-resident.  A wait that exceeds SPIN_LIMIT polls sets
// the sticky error word and makes every CTA return, so a lost arrival can never hang the GPU.
constexpr unsigned SPIN_LIMIT = 4u * 1000u * 1000u;
enum ErrCode { ERR_NONE = 0, ERR_BARRIER_TIMEOUT = 1, ERR_BAD_ARG = 2 };

struct GridBar {
    unsigned* counter;
    unsigned* gen;
    int* err;
    unsigned nblocks;
    unsigned cur;      // generation this CTA expects to leave behind
};

__device__ __forceinline__ bool grid_sync(GridBar& b, int* s_flag) {
    __syncthreads();
    if (threadIdx.x == 0) {
        int ok = 1;
        __threadfence();
        unsigned prev = atomicAdd(b.counter, 1u);
        if (prev == b.nblocks - 1) {
            atomicExch(b.counter, 0u);
            __threadfence();
            st_release(b.gen, b.cur + 1u);
        } else {
            unsigned it = 0;
            while (ld_acquire(b.gen) == b.cur) {
                if (++it > SPIN_LIMIT || ((it & 1023u) == 0 && ld_volatile(b.err) != 0)) {
                    atomicCAS(b.err, 0, (int)ERR_BARRIER_TIMEOUT);
                    ok = 0;
                    break;
                }
            }
        }
        __threadfence();
        *s_flag = ok;
    }
    b.cur += 1u;
    __syncthreads();
    return *s_flag != 0;
}

// ---- legacy tensor-core path (mma.sync m16n8k16 bf16) for the attention products: fragment loads and the MMA ----
__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void* p) {
    const uint32_t a = (uint32_t)__cvta_generic_to_shared(p);
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];" : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(a));
}
__device__ __forceinline__ void ldsm_x4_trans(uint32_t (&r)[4], const void* p) {
    const uint32_t a = (uint32_t)__cvta_generic_to_shared(p);
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];" : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(a));
}
__device__ __forceinline__ void mma_16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                 : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// 16 bytes global -> shared without passing through registers; complete after cp_async_wait_all() + a barrier
__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gsrc) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(smem_dst)), "l"(gsrc) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
    asm volatile("cp.async.commit_group;" ::: "memory");
    asm volatile("cp.async.wait_group 0;" ::: "memory");
}

typedef unsigned long long u64;

// ---- mbarrier / TMA bulk primitives (inline PTX) ----------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_fence_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok) : "r"(bar), "r"(parity) : "memory");
    return ok != 0;
}
__device__ __forceinline__ u64 l2_policy_evict_first() {
    u64 p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}
// 1-D bulk copy global -> this CTA's shared memory, completion counted on `bar`.
// Both addresses and the size are multiples of 16 bytes.  No multicast.
__device__ __forceinline__ void tma_load_1d(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar, u64 policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;"
        ::"r"(dst), "l"(src), "r"(bytes), "r"(bar), "l"(policy) : "memory");
}
// 2-D tiled copy through a tensor map (global -> this CTA's shared memory), completion counted on `bar`.  No multicast.
// x (innermost coordinate) times the element size must be a multiple of 16 bytes.
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const void* tmap, int x, int y, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
        ::"r"(dst), "l"(tmap), "r"(x), "r"(y), "r"(bar) : "memory");
}
// the same copy without a cache hint
__device__ __forceinline__ void bulk_load_1d(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 ::"r"(dst), "l"(src), "r"(bytes), "r"(bar) : "memory");
}

// Programmatic dependent launch: a kernel launched with the programmatic-stream-serialization attribute may start while
// the kernel before it in the stream is still draining; it must call this before it reads or writes anything that
// kernel touches.  Without the attribute the instruction returns at once.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
// Lets the next kernel of the stream be scheduled now instead of when this grid's last block exits: its blocks run whatever
// they do in front of their own pdl_wait() (set-up, loads of constant weights) beside this grid.  Only for small kernels
// whose blocks are all resident at once: a waiting successor holds shared and tensor memory.
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

}  // namespace q35
