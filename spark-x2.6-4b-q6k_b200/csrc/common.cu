// common.cu — host helpers shared by every libspk entry point.
#include <stdarg.h>

#include "common.cuh"
#include "spk.h"

namespace spk {

static thread_local char t_err[512];

const char *last_error() { return t_err; }

int set_error(const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(t_err, sizeof t_err, fmt, ap);
    va_end(ap);
    return -1;
}

int cuda_fail(const char *what, cudaError_t e) { return set_error("%s: %s", what, cudaGetErrorString(e)); }

// One error word per device. Kernels receive its address and set it instead
// of trapping; the host polls it at its sync points.
__device__ int g_dev_err;

static int *g_err_ptr[64];

int *device_error_ptr() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
    if (!g_err_ptr[dev]) {
        void *p = nullptr;
        if (cudaGetSymbolAddress(&p, g_dev_err) != cudaSuccess) return nullptr;
        g_err_ptr[dev] = (int *)p;
    }
    return g_err_ptr[dev];
}

int check_device_error(const char *where) {
    int v = 0;
    cudaError_t e = cudaMemcpyFromSymbol(&v, g_dev_err, sizeof v);
    if (e != cudaSuccess) return cuda_fail(where, e);
    if (v != DEV_OK) {
        int z = 0;
        cudaMemcpyToSymbol(g_dev_err, &z, sizeof z);
        return set_error("%s: device reported %s", where,
                         v == DEV_WAIT_TIMEOUT   ? "a wait that ran out (copy never completed)"
                         : v == DEV_PEER_TIMEOUT ? "a peer that never reached an exchange (tensor-parallel rank missing or stalled)"
                                                 : "an out-of-range index");
    }
    return 0;
}

int sm_count() {
    static int n[64];
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return 148;
    if (!n[dev]) {
        int v = 0;
        if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0) v = 148;
        n[dev] = v;
    }
    return n[dev];
}

size_t smem_optin_max() {
    static size_t v[64];
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return 48 * 1024;
    if (!v[dev]) {
        int x = 0;
        v[dev] = (cudaDeviceGetAttribute(&x, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) == cudaSuccess && x > 0)
                     ? (size_t)x
                     : (size_t)(48 * 1024);
    }
    return v[dev];
}

}  // namespace spk

extern "C" {

/* decode-gpu.cu:23 */
const char *vqg_decode_error(void) { return spk::last_error(); }

const char *spk_last_error(void) { return spk::last_error(); }

int spk_check_device_error(void) { return spk::check_device_error("spk_check_device_error"); }

/* decode-gpu.cu:769-776, for the current device rather than device 0. */
int vqg_device_name(char *out, int n) {
    cudaDeviceProp p;
    memset(&p, 0, sizeof p);
    int dev = 0;
    cudaGetDevice(&dev);
    if (!out || n <= 0) return spk::set_error("device name buffer is empty");
    cudaError_t e = cudaGetDeviceProperties(&p, dev);
    if (e != cudaSuccess) return spk::cuda_fail("device properties", e);
    snprintf(out, (size_t)n, "%s", p.name);
    return 0;
}

/* decode-gpu.cu:780-784 */
int vqg_driver_version(void) {
    int v = 0;
    if (cudaDriverGetVersion(&v) != cudaSuccess) return -1;
    return v;
}

}  // extern "C"
