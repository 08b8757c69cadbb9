// Draft-tree construction around the tree-verify pass: the per-position top-K log-probabilities of the draft model on
// the GPU, and the best-first tree built from them on the host.  Replaces extract_draft_topk (OpenMP over the
// vocabulary on the CPU) and build_ddtree of the reference's driver (models/qwen35_27b/test/test_dflash.cpp:143-207,
// 218-390).
#include <cmath>
#include <queue>
#include <vector>

#include "common.cuh"
#include "runtime.h"

namespace q35 {

constexpr int TOPK_MAX = 16;
constexpr int TOPK_THREADS = 1024;

// One CTA per position: log-sum-exp of logits / T over the vocabulary, then K rounds of arg-max (each round excludes
// everything at or above the previous pick in (value, index) order), so the output is sorted by descending value and,
// among equal values, ascending token id.
__global__ void __launch_bounds__(TOPK_THREADS) draft_topk_kernel(const float* __restrict__ logits, int vocab, int K, float inv_t,
                                                                  float* __restrict__ out_lp, int* __restrict__ out_id) {
    __shared__ float sv[32];
    __shared__ int si[32];
    __shared__ float s_bcast[2];
    __shared__ int s_pick;
    const float* row = logits + (size_t)blockIdx.x * vocab;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    // maximum
    float mx = -INFINITY;
    for (int j = tid; j < vocab; j += TOPK_THREADS) mx = fmaxf(mx, row[j] * inv_t);
    mx = warp_max(mx);
    if (lane == 0) sv[warp] = mx;
    __syncthreads();
    if (warp == 0) { float v = sv[lane]; v = warp_max(v); if (lane == 0) s_bcast[0] = v; }
    __syncthreads();
    mx = s_bcast[0];
    float sm = 0.f;
    for (int j = tid; j < vocab; j += TOPK_THREADS) sm += expf(row[j] * inv_t - mx);
    sm = warp_sum(sm);
    __syncthreads();
    if (lane == 0) sv[warp] = sm;
    __syncthreads();
    if (warp == 0) { float v = sv[lane]; v = warp_sum(v); if (lane == 0) s_bcast[1] = v; }
    __syncthreads();
    const float log_z = mx + logf(s_bcast[1]);
    float prev_v = INFINITY; int prev_i = -1;
    for (int k = 0; k < K; ++k) {
        float best = -INFINITY; int bi = 0x7fffffff;
        for (int j = tid; j < vocab; j += TOPK_THREADS) {
            const float v = row[j] * inv_t;
            const bool after_prev = v < prev_v || (v == prev_v && j > prev_i);
            if (after_prev && (v > best || (v == best && j < bi))) { best = v; bi = j; }
        }
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, best, o); const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (ov > best || (ov == best && oi < bi)) { best = ov; bi = oi; }
        }
        __syncthreads();
        if (lane == 0) { sv[warp] = best; si[warp] = bi; }
        __syncthreads();
        if (warp == 0) {
            best = sv[lane]; bi = si[lane];
            for (int o = 16; o > 0; o >>= 1) {
                const float ov = __shfl_xor_sync(0xffffffffu, best, o); const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
                if (ov > best || (ov == best && oi < bi)) { best = ov; bi = oi; }
            }
            if (lane == 0) {
                s_bcast[0] = best; s_pick = bi;
                out_lp[(size_t)blockIdx.x * K + k] = best - log_z;
                out_id[(size_t)blockIdx.x * K + k] = bi;
            }
        }
        __syncthreads();
        prev_v = s_bcast[0]; prev_i = s_pick;
    }
}

}  // namespace q35

extern "C" int qwen35_b200_draft_topk(const float* logits, int n_positions, int vocab, int k, float temperature, float* out_log_probs,
                                      int* out_token_ids, qwen35_stream_t stream) {
    using namespace q35;
    if (!logits || !out_log_probs || !out_token_ids || n_positions <= 0 || vocab <= 0 || k <= 0 || k > TOPK_MAX || k > vocab) {
        set_error("draft_topk: bad arguments (1 <= k <= %d, k <= vocab)", TOPK_MAX);
        return QWEN35_ERR_BAD_ARG;
    }
    const float inv_t = 1.0f / fmaxf(1e-3f, temperature);
    draft_topk_kernel<<<n_positions, TOPK_THREADS, 0, (cudaStream_t)stream>>>(logits, vocab, k, inv_t, out_log_probs, out_token_ids);
    Q35_CUDA_OK(cudaGetLastError());
    g_launches.fetch_add(1);
    return QWEN35_OK;
}

// Best-first tree over prefixes of the per-depth top-K lists (host code, no GPU work).  Node 0 is the root; nodes are
// numbered in the order they are accepted into the tree, so parents[i] < i.  A candidate is (parent node, depth, rank);
// accepting it adds its next-rank sibling and its rank-0 child as candidates.  With chain_seed the rank-0 chain is
// taken first.  Candidates of equal log-probability are taken in the order they were created.
extern "C" int qwen35_b200_build_ddtree(const float* top_log_probs, const int* top_token_ids, int depth_max, int k, int budget, int chain_seed,
                                        int* token_ids, int* depths, int* parents, unsigned char* visibility) {
    using namespace q35;
    if (!top_log_probs || !top_token_ids || !token_ids || !depths || !parents || depth_max < 0 || k <= 0 || budget < 0) {
        set_error("build_ddtree: bad arguments");
        return -1;
    }
    struct Cand { float logw; long long seq; int parent, depth, rank; };
    struct Worse {
        bool operator()(const Cand& a, const Cand& b) const { return a.logw < b.logw || (a.logw == b.logw && a.seq > b.seq); }
    };
    std::priority_queue<Cand, std::vector<Cand>, Worse> heap;
    long long seq = 0;
    int n = 0;                                  // nodes beside the root
    parents[0] = -1; depths[0] = 0; token_ids[0] = -1;
    auto lp = [&](int d, int r) { return top_log_probs[(size_t)(d - 1) * k + r]; };
    auto add = [&](int parent, int depth, int rank) {
        ++n;
        token_ids[n] = top_token_ids[(size_t)(depth - 1) * k + rank];
        depths[n] = depth; parents[n] = parent;
        return n;
    };
    if (budget > 0 && depth_max > 0) {
        if (chain_seed) {
            float cum = 0.f;
            int prev = 0;
            for (int d = 1; d <= depth_max && n < budget; ++d) {
                cum += lp(d, 0);
                const int cur = add(prev, d, 0);
                if (k > 1) heap.push(Cand{cum - lp(d, 0) + lp(d, 1), seq++, prev, d, 1});
                prev = cur;
            }
        } else {
            heap.push(Cand{lp(1, 0), seq++, 0, 1, 0});
        }
        while (!heap.empty() && n < budget) {
            const Cand c = heap.top();
            heap.pop();
            const int cur = add(c.parent, c.depth, c.rank);
            if (c.rank + 1 < k) heap.push(Cand{c.logw - lp(c.depth, c.rank) + lp(c.depth, c.rank + 1), seq++, c.parent, c.depth, c.rank + 1});
            if (c.depth < depth_max) heap.push(Cand{c.logw + lp(c.depth + 1, 0), seq++, cur, c.depth + 1, 0});
        }
    }
    if (visibility) {                           // ancestor-or-self matrix, (1 + n)^2 row-major
        const int N = n + 1;
        for (int i = 0; i < N; ++i) {
            for (int j = 0; j < N; ++j) visibility[(size_t)i * N + j] = (i > 0 && j < i) ? visibility[(size_t)parents[i] * N + j] : 0;
            visibility[(size_t)i * N + i] = 1;
        }
    }
    return n;
}
