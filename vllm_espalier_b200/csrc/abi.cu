// Library-wide C ABI pieces: version, per-thread error messages, the device status word, SM counts.
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdlib>
#include <cstdio>
#include <mutex>

#include "common.cuh"
#include "host.hpp"

namespace esp {

int status_dense(int reset);   // one reader per translation unit that has device waits
int status_route(int reset);
int status_moe(int reset);
int status_ep(int reset);

namespace {
thread_local char t_msg[512] = "";
}

int set_error(int code, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(t_msg, sizeof(t_msg), fmt, ap);
    va_end(ap);
    return code;
}

int ok() {
    t_msg[0] = 0;
    return ESP_OK;
}

bool pdl_enabled() {
    static const bool on = [] {
        const char* v = getenv("ESPALIER_PDL");
        return !(v && v[0] == '0');
    }();
    return on;
}

int device_sms() {
    static int cache[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    if (!cache[dev]) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
        cache[dev] = n;
    }
    return cache[dev];
}

}  // namespace esp

extern "C" {

int esp_version(void) { return 100; }

const char* esp_last_error(void) { return esp::t_msg; }

int esp_sm_count(void) { return esp::device_sms(); }

int esp_device_status(int* status, int reset) {
    if (!status) return esp::set_error(ESP_ERR_INVALID, "esp_device_status: status is NULL");
    int v = 0;
    for (int (*rd)(int) : {esp::status_dense, esp::status_route, esp::status_moe, esp::status_ep}) {
        const int s = rd(reset);
        if (s < 0) return esp::set_error(ESP_ERR_CUDA, "esp_device_status: %s", cudaGetErrorString(cudaGetLastError()));
        if (!v) v = s;
    }
    *status = v;
    return esp::ok();
}

}  // extern "C"
