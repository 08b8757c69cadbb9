// Per-device workspace, sticky status word and error reporting for libqwen35_b200.
#include "runtime.h"

#include <cstdarg>
#include <cstdio>
#include <mutex>


namespace q35 {

static constexpr int MAX_DEVICES = 64;
static void* g_ws[MAX_DEVICES] = {};
static int g_sms[MAX_DEVICES] = {};
static int* g_extra_status[MAX_DEVICES] = {};
static std::mutex g_mu;
static thread_local char g_err[512] = "";
std::atomic<long long> g_launches{0};
bool g_pdl_launch = false;
bool g_pdl_early = false;

void set_error(const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof(g_err), fmt, ap);
    va_end(ap);
}

void* get_workspace() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= MAX_DEVICES) {
        set_error("no current CUDA device");
        return nullptr;
    }
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_ws[dev]) {
        void* p = nullptr;
        cudaError_t e = cudaMalloc(&p, workspace_bytes());
        if (e == cudaSuccess) e = cudaMemset(p, 0, workspace_bytes());
        if (e != cudaSuccess) {
            set_error("workspace allocation failed: %s", cudaGetErrorString(e));
            return nullptr;
        }
        g_ws[dev] = p;
    }
    return g_ws[dev];
}

void register_status_word(int* dev_ptr) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= MAX_DEVICES) return;
    std::lock_guard<std::mutex> lk(g_mu);
    g_extra_status[dev] = dev_ptr;
}

int device_sm_count() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= MAX_DEVICES) return 0;
    if (!g_sms[dev]) cudaDeviceGetAttribute(&g_sms[dev], cudaDevAttrMultiProcessorCount, dev);
    return g_sms[dev];
}

}  // namespace q35

// Status words that exist on the current device: the regular workspace's (only if some earlier call already
// allocated it) and the one registered for the static scratch.  Reading the status never creates either.
static int existing_status_words(int* out[2]) {
    int dev = 0, n = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= q35::MAX_DEVICES) return 0;
    std::lock_guard<std::mutex> lk(q35::g_mu);
    if (q35::g_ws[dev]) out[n++] = (int*)q35::g_ws[dev];
    if (q35::g_extra_status[dev]) out[n++] = q35::g_extra_status[dev];
    return n;
}

extern "C" int qwen35_b200_status(qwen35_stream_t stream) {
    using namespace q35;
    int* words[2];
    const int n = existing_status_words(words);
    int err[2] = {0, 0};
    for (int i = 0; i < n; ++i)
        Q35_CUDA_OK(cudaMemcpyAsync(&err[i], words[i], sizeof(int), cudaMemcpyDeviceToHost, (cudaStream_t)stream));
    Q35_CUDA_OK(cudaStreamSynchronize((cudaStream_t)stream));
    const int e = err[0] ? err[0] : err[1];
    if (e) set_error("device status %d (%s)", e, e == 1 ? "a bounded device-side wait ran out" : "bad argument seen on device");
    return e;
}

extern "C" int qwen35_b200_clear_status(qwen35_stream_t stream) {
    using namespace q35;
    int* words[2];
    const int n = existing_status_words(words);
    for (int i = 0; i < n; ++i) Q35_CUDA_OK(cudaMemsetAsync(words[i], 0, sizeof(int), (cudaStream_t)stream));
    return QWEN35_OK;
}

/* Address of the library-allocated workspace of the current device, or NULL while no call has created it (tests). */
extern "C" const void* qwen35_b200_workspace_if_any(void) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= q35::MAX_DEVICES) return nullptr;
    std::lock_guard<std::mutex> lk(q35::g_mu);
    return q35::g_ws[dev];
}

extern "C" long long qwen35_b200_launch_count(void) { return q35::g_launches.load(); }

extern "C" const char* qwen35_b200_last_error(void) { return q35::g_err; }
