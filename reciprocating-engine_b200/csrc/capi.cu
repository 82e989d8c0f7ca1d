// Error plumbing, version and device discovery of the C ABI.
#include <cstdio>
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

// minor 2: reng_model_desc.qk_norm, reng_layer_weights.qn / kn / no_rope
extern "C" int reng_version(void) { return (0 << 16) | 3; }

extern "C" int reng_device_count(int* count) {
    RENG_CHECK_ARG(count != nullptr, "reng_device_count: count is NULL");
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    *count = 0;
    if (e == cudaErrorNoDevice || e == cudaErrorInsufficientDriver) {
        cudaGetLastError();
        return RENG_OK;  // no devices here: an empty enumeration
    }
    if (e != cudaSuccess)
        return reng::fail(RENG_E_CUDA, std::string("cudaGetDeviceCount: ") + cudaGetErrorString(e));
    *count = n;
    return RENG_OK;
}

extern "C" int reng_device_info_get(int device, reng_device_info* out) {
    RENG_CHECK_ARG(out != nullptr, "reng_device_info_get: out is NULL");
    int n = 0;
    if (reng_device_count(&n) != RENG_OK) return RENG_E_CUDA;
    RENG_CHECK_ARG(device >= 0 && device < n, "reng_device_info_get: device " + std::to_string(device) +
                                                  " of " + std::to_string(n));
    cudaDeviceProp p{};
    RENG_CUDA_TRY(cudaGetDeviceProperties(&p, device));
    *out = reng_device_info{};
    out->ordinal = device;
    snprintf(out->name, sizeof(out->name), "%s", p.name);
    RENG_CUDA_TRY(cudaDeviceGetPCIBusId(out->pci_bus_id, (int)sizeof(out->pci_bus_id), device));
    out->total_bytes = (uint64_t)p.totalGlobalMem;
    out->sm_count = p.multiProcessorCount;
    out->cc_major = p.major;
    out->cc_minor = p.minor;
    return RENG_OK;
}
