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

#define Q35_CUDA_OK(expr)                                                         \
    do {                                                                          \
        cudaError_t e__ = (expr);                                                 \
        if (e__ != cudaSuccess) {                                                 \
            q35::set_error("%s failed: %s", #expr, cudaGetErrorString(e__));      \
            return QWEN35_ERR_CUDA;                                               \
        }                                                                         \
    } while (0)

}  // namespace q35
