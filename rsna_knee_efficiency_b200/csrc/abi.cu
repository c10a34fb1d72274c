// abi.cu -- the extern "C" entry points of libdn8b200.so (declared in include/dn8.h).
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <unordered_map>

#include "dn8_kernels.h"

namespace {

thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return code;
}

int cuda_fail(cudaError_t e, const char* what) {
    return fail(DN8_ECUDA, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

// SM count of the current device, cached per device.
int current_sms(int* out) {
    static std::mutex mu;
    static std::unordered_map<int, int> cache;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
    std::lock_guard<std::mutex> lk(mu);
    auto it = cache.find(dev);
    if (it == cache.end()) {
        int sms = 0;
        e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute");
        it = cache.emplace(dev, sms).first;
    }
    *out = it->second;
    return DN8_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

extern "C" {

const char* dn8_last_error(void) { return g_last_error.c_str(); }

int dn8_device_sms(int device) {
    int sms = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess) return 0;
    return sms;
}

int dn8_conv1(const dn8_conv1_args* a, dn8_stream stream) {
    if (a == nullptr) return fail(DN8_EINVAL, "dn8_conv1: null arguments");
    if (a->G < 1 || a->G0 < 1 || a->G0 > a->G || a->N < 1 || a->HW < 1)
        return fail(DN8_EINVAL, "dn8_conv1: bad geometry G0=%d G=%d N=%d HW=%d", a->G0, a->G, a->N, a->HW);
    if (static_cast<long long>(a->N) * a->HW * 128 >= (1ll << 31))
        return fail(DN8_EINVAL, "dn8_conv1: N*HW*128 exceeds 2^31");
    if (!aligned16(a->in0) || !aligned16(a->seg) || !aligned16(a->w) || !aligned16(a->ab) ||
        !aligned16(a->out) || a->gd == nullptr)
        return fail(DN8_EINVAL, "dn8_conv1: pointers must be non-null and 16-byte aligned");
    int sms = 0;
    if (int s = current_sms(&sms)) return s;
    cudaError_t e = dn8::launch_conv1(*a, sms, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? DN8_OK : cuda_fail(e, "dn8_conv1 launch");
}

int dn8_conv2(const dn8_conv2_args* a, dn8_stream stream) {
    if (a == nullptr) return fail(DN8_EINVAL, "dn8_conv2: null arguments");
    if (a->N < 1 || a->H < 1 || a->W < 1 || a->W > 128)
        return fail(DN8_EINVAL, "dn8_conv2: unsupported geometry N=%d H=%d W=%d (W <= 128)", a->N, a->H, a->W);
    if (!aligned16(a->x) || !aligned16(a->w) || !aligned16(a->out) || a->sc == nullptr)
        return fail(DN8_EINVAL, "dn8_conv2: pointers must be non-null and 16-byte aligned");
    dn8::Conv2Plan plan;
    cudaError_t e = dn8::prepare_conv2(&plan, *a);
    if (e != cudaSuccess) return cuda_fail(e, "dn8_conv2 tensor map");
    int sms = 0;
    if (int s = current_sms(&sms)) return s;
    e = dn8::launch_conv2(plan, *a, sms, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? DN8_OK : cuda_fail(e, "dn8_conv2 launch");
}

}  // extern "C"
