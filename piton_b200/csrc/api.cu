// Runtime half of the C ABI: error state, device set-up, memory helpers and a
// bounded stream wait.  The B200 counterpart of pi/runtime/piton_rt.c (mailbox
// allocation, launch with a 20 s timeout, perf counters).
#include <atomic>
#include <chrono>
#include <string>
#include <thread>

#include "common.cuh"

namespace piton {

static thread_local std::string g_last_error;

int set_error(int code, const char *fmt, ...) {
    char buf[1024];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return code;
}

void clear_error() { g_last_error.clear(); }

static std::atomic<uint64_t> g_launches{0};

void count_launches(int n) { g_launches.fetch_add((uint64_t)n, std::memory_order_relaxed); }

int check_launch(const char *what, int launches) {
    count_launches(launches);
    cudaError_t err = cudaGetLastError();
    if (err != cudaSuccess) return set_error(PITON_B200_ECUDA, "%s: %s", what, cudaGetErrorString(err));
    return PITON_B200_OK;
}

int num_sms() {
    static int cache[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return 148;
    if (cache[dev] == 0) {
        int n = 0;
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        cache[dev] = n > 0 ? n : 148;
    }
    return cache[dev];
}

}  // namespace piton

using namespace piton;

extern "C" {

int piton_b200_abi_version(void) { return PITON_B200_ABI_VERSION; }

uint64_t piton_b200_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

const char *piton_b200_last_error(void) { return g_last_error.c_str(); }

int piton_b200_init(int device) {
    int count = 0;
    PITON_CUDA(cudaGetDeviceCount(&count));
    PITON_REQUIRE(device >= 0 && device < count, "device %d out of range (%d devices)", device, count);
    PITON_CUDA(cudaSetDevice(device));
    PITON_CUDA(cudaFree(nullptr));     // creates the primary context
    cudaDeviceProp prop;
    PITON_CUDA(cudaGetDeviceProperties(&prop, device));
    if (prop.major != 10)
        return set_error(PITON_B200_ENOTSUP, "device %d is sm_%d%d; this library is built for sm_100a",
                         device, prop.major, prop.minor);
    return PITON_B200_OK;
}

int piton_b200_device_count(int *count) {
    PITON_REQUIRE(count != nullptr, "count is NULL");
    PITON_CUDA(cudaGetDeviceCount(count));
    return PITON_B200_OK;
}

int piton_b200_get_device(int *device) {
    PITON_REQUIRE(device != nullptr, "device is NULL");
    PITON_CUDA(cudaGetDevice(device));
    return PITON_B200_OK;
}

int piton_b200_malloc(uint64_t *ptr, size_t bytes) {
    PITON_REQUIRE(ptr != nullptr, "ptr is NULL");
    void *p = nullptr;
    cudaError_t err = cudaMalloc(&p, bytes ? bytes : 1);
    if (err != cudaSuccess)
        return set_error(PITON_B200_ENOMEM, "cudaMalloc(%zu): %s", bytes, cudaGetErrorString(err));
    *ptr = reinterpret_cast<uint64_t>(p);
    return PITON_B200_OK;
}

int piton_b200_free(uint64_t ptr) {
    PITON_CUDA(cudaFree(reinterpret_cast<void *>(ptr)));
    return PITON_B200_OK;
}

int piton_b200_memcpy_h2d(uint64_t dst, const void *src, size_t bytes, void *stream) {
    PITON_REQUIRE(bytes == 0 || (dst && src), "NULL pointer");
    PITON_CUDA(cudaMemcpyAsync(reinterpret_cast<void *>(dst), src, bytes, cudaMemcpyHostToDevice, as_stream(stream)));
    return PITON_B200_OK;
}

int piton_b200_memcpy_d2h(void *dst, uint64_t src, size_t bytes, void *stream) {
    PITON_REQUIRE(bytes == 0 || (dst && src), "NULL pointer");
    PITON_CUDA(cudaMemcpyAsync(dst, reinterpret_cast<const void *>(src), bytes, cudaMemcpyDeviceToHost, as_stream(stream)));
    return PITON_B200_OK;
}

int piton_b200_memset(uint64_t dst, int value, size_t bytes, void *stream) {
    PITON_CUDA(cudaMemsetAsync(reinterpret_cast<void *>(dst), value, bytes, as_stream(stream)));
    return PITON_B200_OK;
}

int piton_b200_ipc_handle(uint64_t ptr, void *handle) {
    PITON_REQUIRE(ptr && handle, "NULL pointer");
    cudaIpcMemHandle_t h;
    PITON_CUDA(cudaIpcGetMemHandle(&h, reinterpret_cast<void *>(ptr)));
    memcpy(handle, &h, sizeof h);
    return PITON_B200_OK;
}

int piton_b200_ipc_open(const void *handle, uint64_t *ptr) {
    PITON_REQUIRE(ptr && handle, "NULL pointer");
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof h);
    void *p = nullptr;
    PITON_CUDA(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
    *ptr = reinterpret_cast<uint64_t>(p);
    return PITON_B200_OK;
}

int piton_b200_ipc_close(uint64_t ptr) {
    PITON_CUDA(cudaIpcCloseMemHandle(reinterpret_cast<void *>(ptr)));
    return PITON_B200_OK;
}

int piton_b200_stream_wait(void *stream, double timeout_s) {
    using clock = std::chrono::steady_clock;
    auto deadline = clock::now() + std::chrono::duration<double>(timeout_s);
    int spins = 0;
    for (;;) {
        cudaError_t err = cudaStreamQuery(as_stream(stream));
        if (err == cudaSuccess) return PITON_B200_OK;
        if (err != cudaErrorNotReady)
            return set_error(PITON_B200_ECUDA, "stream wait: %s", cudaGetErrorString(err));
        if (clock::now() >= deadline)
            return set_error(PITON_B200_ETIMEOUT, "stream not idle after %.3f s", timeout_s);
        if (++spins > 64) std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
}

}  // extern "C"
