// Host-side runtime shared by the launchers: per-device workspace, status word, error text.
#pragma once

#include <cuda_runtime.h>

#include <atomic>

#include "../../include/qwen35_b200.h"

namespace q35 {

// Workspace of the current device; allocated and zeroed on first use (never inside a capture).
// Its first int is the sticky device status word.  Returns nullptr and records an error string
// on failure.
void* get_workspace();
size_t workspace_bytes();      // defined next to the kernels that lay the workspace out
// Additional device status words (first int of another scratch area) that qwen35_b200_status() must read too.
void register_status_word(int* dev_ptr);

int device_sm_count();
void set_error(const char* fmt, ...);
extern std::atomic<long long> g_launches;
// set by a caller whose every kernel begins with pdl_wait(): the GEMM launchers then add the programmatic-stream-
// serialization attribute to their launches (the GEMM kernels call pdl_wait() after their prologue)
extern bool g_pdl_launch;
extern bool g_pdl_early;      // the bf16 GEMM loads its first weight tiles in front of its dependency wait and releases its successor at its start

// cudaFuncSetAttribute acts on the current device only, so a launcher's "attribute set" flag is kept per device.
// Two host threads that race here both set the attribute, which is harmless.
struct PerDeviceOnce {
    std::atomic<bool> done[64] = {};
    static int slot() { int d = 0; return cudaGetDevice(&d) == cudaSuccess ? (d & 63) : 0; }
    bool pending() const { return !done[slot()].load(std::memory_order_acquire); }
    void mark() { done[slot()].store(true, std::memory_order_release); }
};

#define Q35_CUDA_OK(expr)                                                         \
    do {                                                                          \
        cudaError_t e__ = (expr);                                                 \
        if (e__ != cudaSuccess) {                                                 \
            q35::set_error("%s failed: %s", #expr, cudaGetErrorString(e__));      \
            return QWEN35_ERR_CUDA;                                               \
        }                                                                         \
    } while (0)

// launch with the programmatic-stream-serialization attribute: the kernel may be scheduled while its predecessor in the
// stream drains.  Only for kernels that begin with pdl_wait() (common.cuh).  Also valid under stream capture.
template <typename... KArgs, typename... Args>
static inline cudaError_t pdl_launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream, Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid; cfg.blockDim = block; cfg.dynamicSmemBytes = smem; cfg.stream = stream;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at; cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}
struct PdlGuard {          // while alive, the GEMM launchers add the attribute too
    PdlGuard() { g_pdl_launch = true; }
    ~PdlGuard() { g_pdl_launch = false; }
};
struct PdlEarlyGuard {     // for passes of short kernels (a decode step, a draft forward), where the B operand is always a weight matrix
    PdlEarlyGuard() { g_pdl_early = true; }
    ~PdlEarlyGuard() { g_pdl_early = false; }
};

}  // namespace q35
