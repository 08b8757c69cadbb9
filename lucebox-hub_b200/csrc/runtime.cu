// Per-device workspace, sticky status word and error reporting for libqwen35_b200.
#include "runtime.h"

#include <cstdarg>
#include <cstdio>
#include <mutex>


namespace q35 {

static constexpr int MAX_DEVICES = 64;
static void* g_ws[MAX_DEVICES] = {};
static int g_sms[MAX_DEVICES] = {};
static std::mutex g_mu;
static thread_local char g_err[512] = "";
std::atomic<long long> g_launches{0};
bool g_pdl_launch = false;

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

static int* g_extra_status[MAX_DEVICES] = {};

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

extern "C" int qwen35_b200_status(qwen35_stream_t stream) {
    using namespace q35;
    void* ws = get_workspace();
    if (!ws) return QWEN35_ERR_CUDA;
    int err = 0;
    Q35_CUDA_OK(cudaMemcpyAsync(&err, ws, sizeof(int), cudaMemcpyDeviceToHost, (cudaStream_t)stream));
    int dev = 0;
    int err2 = 0;
    if (cudaGetDevice(&dev) == cudaSuccess && dev >= 0 && dev < MAX_DEVICES && g_extra_status[dev])
        Q35_CUDA_OK(cudaMemcpyAsync(&err2, g_extra_status[dev], sizeof(int), cudaMemcpyDeviceToHost, (cudaStream_t)stream));
    Q35_CUDA_OK(cudaStreamSynchronize((cudaStream_t)stream));
    if (!err) err = err2;
    if (err) set_error("device status %d (%s)", err, err == 1 ? "a bounded device-side wait ran out" : "bad argument seen on device");
    return err;
}

extern "C" int qwen35_b200_clear_status(qwen35_stream_t stream) {
    using namespace q35;
    void* ws = get_workspace();
    if (!ws) return QWEN35_ERR_CUDA;
    Q35_CUDA_OK(cudaMemsetAsync(ws, 0, 256, (cudaStream_t)stream));
    int dev = 0;
    if (cudaGetDevice(&dev) == cudaSuccess && dev >= 0 && dev < MAX_DEVICES && g_extra_status[dev])
        Q35_CUDA_OK(cudaMemsetAsync(g_extra_status[dev], 0, sizeof(int), (cudaStream_t)stream));
    return QWEN35_OK;
}

extern "C" long long qwen35_b200_launch_count(void) { return q35::g_launches.load(); }

extern "C" const char* qwen35_b200_last_error(void) { return q35::g_err; }
