// Error plumbing, version and device discovery of the C ABI.
#include <mutex>
#include <string>
#include <vector>

#include "common.cuh"

namespace reng {

static thread_local std::string g_last_error;

void set_error(const std::string& msg) { g_last_error = msg; }

int fail(int code, const std::string& msg) {
    set_error(msg);
    return code;
}

int num_sms(int device) {
    static std::mutex mu;
    static std::vector<int> cache;
    std::lock_guard<std::mutex> lock(mu);
    if (device < 0) return 148;
    if ((int)cache.size() <= device) cache.resize(device + 1, 0);
    if (cache[device] == 0) {
        int v = 0;
        if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, device) != cudaSuccess ||
            v <= 0)
            v = 148;
        cache[device] = v;
    }
    return cache[device];
}

}  // namespace reng

extern "C" const char* reng_last_error(void) { return reng::g_last_error.c_str(); }

extern "C" int reng_version(void) { return (0 << 16) | 1; }

extern "C" int reng_device_count(int* count) {
    RENG_CHECK_ARG(count != nullptr, "reng_device_count: count is NULL");
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess) {
        *count = 0;
        return reng::fail(RENG_E_CUDA, std::string("cudaGetDeviceCount: ") + cudaGetErrorString(e));
    }
    *count = n;
    return RENG_OK;
}
