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

namespace dn8 {
void set_last_error(const char* msg) { g_last_error = msg ? msg : ""; }
}  // namespace dn8

extern "C" {

const char* dn8_last_error(void) { return g_last_error.c_str(); }

int dn8_device_sms(int device) {
    int sms = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess) return 0;
    return sms;
}

int dn8_conv1(const dn8_conv1_args* a, dn8_stream stream) {
    if (a == nullptr) return fail(DN8_EINVAL, "dn8_conv1: null arguments");
    const bool tiled = a->tile_groups != 0;
    if (a->G < 1 || a->N < 1 || a->HW < 1 || (!tiled && (a->G0 < 1 || a->G0 > a->G)) ||
        (tiled && a->tile_groups < a->G))
        return fail(DN8_EINVAL, "dn8_conv1: bad geometry G0=%d G=%d N=%d HW=%d tile_groups=%d", a->G0, a->G, a->N,
                    a->HW, a->tile_groups);
    if (!dn8::conv1_supported(a->G))
        return fail(DN8_EINVAL, "dn8_conv1: G=%d K groups exceed the supported 70 (2240 input channels)", a->G);
    if (static_cast<long long>(a->N) * a->HW * 128 >= (1ll << 31) ||
        (tiled && static_cast<long long>((a->N * a->HW + 127) / 128) * a->tile_groups * 4096 >= (1ll << 40)))
        return fail(DN8_EINVAL, "dn8_conv1: N*HW*128 exceeds 2^31");
    if (!aligned16(a->in0) || (!tiled && !aligned16(a->seg)) || !aligned16(a->w) || !aligned16(a->ab) ||
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
    if (a->tile_groups < 0 || (a->tile_groups > 0 && (a->group < 0 || a->group >= a->tile_groups)))
        return fail(DN8_EINVAL, "dn8_conv2: group %d outside the tile-major store's %d groups", a->group,
                    a->tile_groups);
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

int dn8_trans(const dn8_trans_args* a, dn8_stream stream) {
    if (a == nullptr) return fail(DN8_EINVAL, "dn8_trans: null arguments");
    if (a->G < 8 || a->G % 8 || a->G0 < 1 || a->G0 > a->G || a->N < 1 || a->H < 2 || a->W < 2 || a->H % 2 ||
        a->W % 2)
        return fail(DN8_EINVAL, "dn8_trans: bad geometry G0=%d G=%d N=%d H=%d W=%d", a->G0, a->G, a->N, a->H, a->W);
    if (a->G * 16 > 640) return fail(DN8_EINVAL, "dn8_trans: c_out %d > 640", a->G * 16);
    if (a->tile_groups < 0 || (a->tile_groups > 0 && a->tile_groups < a->G) || a->out_tile_groups < 0 ||
        (a->out_tile_groups > 0 && a->out_tile_groups < a->G / 2))
        return fail(DN8_EINVAL, "dn8_trans: tile-major stores of %d (in) / %d (out) groups cannot hold %d / %d",
                    a->tile_groups, a->out_tile_groups, a->G, a->G / 2);
    if (!aligned16(a->in0) || (a->tile_groups == 0 && !aligned16(a->seg)) || !aligned16(a->w) ||
        !aligned16(a->ab) || !aligned16(a->out) || a->gd == nullptr)
        return fail(DN8_EINVAL, "dn8_trans: pointers must be non-null and 16-byte aligned");
    int sms = 0;
    if (int s = current_sms(&sms)) return s;
    cudaError_t e = dn8::launch_trans(*a, sms, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? DN8_OK : cuda_fail(e, "dn8_trans launch");
}

// [rows][32] tile -> tcgen05 K-major 32-byte-swizzle layout: 16-byte half h of row r goes to
// r * 32 + ((h ^ ((r >> 2) & 1)) << 4).
static void swizzle32_tile(const int8_t* src, int rows, uint8_t* dst) {
    for (int r = 0; r < rows; ++r)
        for (int h = 0; h < 2; ++h)
            std::memcpy(dst + r * 32 + ((h ^ ((r >> 2) & 1)) << 4), src + r * 32 + h * 16, 16);
}

int dn8_prepare_conv1_weights(const int8_t* w1, int32_t G, uint8_t* out) {
    if (w1 == nullptr || out == nullptr || G < 1) return fail(DN8_EINVAL, "dn8_prepare_conv1_weights: bad arguments");
    for (int g = 0; g < G; ++g) swizzle32_tile(w1 + static_cast<size_t>(g) * 4096, 128, out + static_cast<size_t>(g) * 4096);
    return DN8_OK;
}

int dn8_prepare_trans_weights(const int8_t* tw, int32_t G, int32_t cout, uint8_t* out) {
    if (tw == nullptr || out == nullptr || G < 1 || cout < 128 || cout % 128)
        return fail(DN8_EINVAL, "dn8_prepare_trans_weights: bad arguments");
    const int nc = dn8::trans_chunk(cout), nchunks = (cout + nc - 1) / nc;
    // [nchunks][G][w rows][32]: chunk c holds output channels c * nc .. c * nc + w - 1,
    // w = min(nc, cout - c * nc), and starts at byte G * 32 * c * nc
    for (int c = 0; c < nchunks; ++c) {
        const int w = cout - c * nc < nc ? cout - c * nc : nc;
        for (int g = 0; g < G; ++g)
            swizzle32_tile(tw + (static_cast<size_t>(g) * cout + static_cast<size_t>(c) * nc) * 32, w,
                           out + static_cast<size_t>(G) * 32 * c * nc + static_cast<size_t>(g) * w * 32);
    }
    return DN8_OK;
}

int dn8_stem(const dn8_stem_args* a, dn8_stream stream) {
    if (a == nullptr) return fail(DN8_EINVAL, "dn8_stem: null arguments");
    if (a->N < 1 || a->H < 4 || a->W < 4 || a->H % 4 || a->W % 4 || a->W > 512)
        return fail(DN8_EINVAL, "dn8_stem: unsupported geometry N=%d H=%d W=%d (multiples of 4, W <= 512)", a->N,
                    a->H, a->W);
    if (a->x == nullptr || !aligned16(a->w) || a->kc == nullptr || !aligned16(a->out) || (a->x_u8 && a->src == nullptr))
        return fail(DN8_EINVAL, "dn8_stem: bad pointers");
    if (a->tile_groups < 0 || a->tile_groups == 1)
        return fail(DN8_EINVAL, "dn8_stem: a tile-major store needs at least the 2 groups the stem writes");
    int sms = 0;
    if (int s = current_sms(&sms)) return s;
    cudaError_t e = dn8::launch_stem(*a, sms, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? DN8_OK : cuda_fail(e, "dn8_stem launch");
}

int dn8_head(const dn8_head_args* a, dn8_stream stream) {
    if (a == nullptr) return fail(DN8_EINVAL, "dn8_head: null arguments");
    if (a->G < 1 || a->G > 72 || a->G0 < 1 || a->G0 > a->G || a->N < 1 || a->HW < 1 || a->n_out < 0 ||
        a->n_out > 64 || a->tile_groups < 0 || (a->tile_groups > 0 && a->tile_groups < a->G))
        return fail(DN8_EINVAL, "dn8_head: bad geometry (G <= 72, n_out <= 64)");
    if (!aligned16(a->in0) || (a->tile_groups == 0 && !aligned16(a->seg)) || a->fab == nullptr)
        return fail(DN8_EINVAL, "dn8_head: bad pointers");
    if (a->hw != nullptr && (a->hb == nullptr || a->logits == nullptr))
        return fail(DN8_EINVAL, "dn8_head: head without bias or logits buffer");
    if (a->view_logits != nullptr && a->hw == nullptr)
        return fail(DN8_EINVAL, "dn8_head: view_logits need the head (hw, hb, logits)");
    if (a->view_logits != nullptr && (a->per_view < 1 || a->N % a->per_view || a->tickets == nullptr))
        return fail(DN8_EINVAL, "dn8_head: views need per_view dividing N and a ticket array");
    cudaError_t e = dn8::launch_head(*a, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? DN8_OK : cuda_fail(e, "dn8_head launch");
}

int dn8_zoom(const dn8_zoom_args* a, dn8_stream stream) {
    if (a == nullptr) return fail(DN8_EINVAL, "dn8_zoom: null arguments");
    if (a->N < 1 || a->H < 2 || a->W < 16 || a->W % 16 || !(a->scale >= 0.25) || a->planes == nullptr || a->src == nullptr ||
        a->out == nullptr)
        return fail(DN8_EINVAL, "dn8_zoom: bad arguments N=%d H=%d W=%d scale=%g", a->N, a->H, a->W,
                    a->scale);
    int sms = 0;
    if (int s = current_sms(&sms)) return s;
    cudaError_t e = dn8::launch_zoom(*a, sms, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? DN8_OK : cuda_fail(e, "dn8_zoom launch");
}

int dn8_head_noalloc(const dn8_head_args* a, dn8_stream stream) {
    if (a == nullptr) return fail(DN8_EINVAL, "dn8_head_noalloc: null arguments");
    if (a->view_logits != nullptr && a->per_view >= 1 && a->N % a->per_view == 0 &&
        a->N / a->per_view > DN8_HEAD_SCRATCH_VIEWS)
        return fail(DN8_EINVAL, "dn8_head_noalloc: %d views (N / per_view), the built-in scratch holds %d",
                    a->N / a->per_view, DN8_HEAD_SCRATCH_VIEWS);
    if (a->tickets != nullptr)
        return fail(DN8_EINVAL, "dn8_head_noalloc: tickets must be NULL (the built-in scratch is used)");
    if (a->G < 1 || a->G > 72 || a->G0 < 1 || a->G0 > a->G || a->N < 1 || a->HW < 1 || a->n_out < 0 ||
        a->n_out > 64 || a->tile_groups < 0 || (a->tile_groups > 0 && a->tile_groups < a->G))
        return fail(DN8_EINVAL, "dn8_head_noalloc: bad geometry (G <= 72, n_out <= 64)");
    if (!aligned16(a->in0) || (a->tile_groups == 0 && !aligned16(a->seg)) || a->fab == nullptr)
        return fail(DN8_EINVAL, "dn8_head_noalloc: bad pointers");
    if (a->hw != nullptr && (a->hb == nullptr || a->logits == nullptr))
        return fail(DN8_EINVAL, "dn8_head_noalloc: head without bias or logits buffer");
    if (a->view_logits != nullptr && a->hw == nullptr)
        return fail(DN8_EINVAL, "dn8_head_noalloc: view_logits need the head (hw, hb, logits)");
    if (a->view_logits != nullptr && (a->per_view < 1 || a->N % a->per_view))
        return fail(DN8_EINVAL, "dn8_head_noalloc: views need per_view dividing N");
    dn8_head_args args = *a;
    if (args.view_logits != nullptr) {
        cudaError_t e = dn8::head_scratch_tickets(&args.tickets);
        if (e != cudaSuccess) return cuda_fail(e, "dn8_head_noalloc scratch address");
    }
    cudaError_t e = dn8::launch_head(args, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? DN8_OK : cuda_fail(e, "dn8_head_noalloc launch");
}

int dn8_test_inject_wait_fault(int32_t fault, int64_t wait_limit_cycles) {
    if (fault < 0 || fault > 1 || wait_limit_cycles < 0 || (fault == 1 && wait_limit_cycles == 0))
        return fail(DN8_EINVAL, "dn8_test_inject_wait_fault: fault 0 or 1 (with a wait limit > 0)");
    dn8::arm_wait_fault(fault, wait_limit_cycles);
    return DN8_OK;
}

int dn8_prepare_stem_weights(const int8_t* w8, uint8_t* out) {
    if (w8 == nullptr || out == nullptr) return fail(DN8_EINVAL, "dn8_prepare_stem_weights: bad arguments");
    // S_w8 [64][176] (k = (ch * 7 + ky) * 8 + kx') -> 7 K steps, one per kernel row ky, of
    // [64 rows][32 B] = [ch 0 kx' 0..7 | ch 1 | ch 2 | 8 zero bytes], 32B-swizzled
    int8_t tile[64 * 32];
    for (int ky = 0; ky < 7; ++ky) {
        for (int o = 0; o < 64; ++o)
            for (int c = 0; c < 32; ++c) {
                const int ch = c / 8, kx = c % 8;
                tile[o * 32 + c] = ch < 3 ? w8[o * 176 + (ch * 7 + ky) * 8 + kx] : 0;
            }
        swizzle32_tile(tile, 64, out + ky * 2048);
    }
    return DN8_OK;
}

int dn8_prepare_conv2_weights(const int8_t* w2k, uint8_t* out) {
    if (w2k == nullptr || out == nullptr) return fail(DN8_EINVAL, "dn8_prepare_conv2_weights: bad arguments");
    // w2k [cblk][tap][o][32] -> [dy][cblk][half][dx * 32 + o][16] (tap = 3 dy + dx)
    for (int blk = 0; blk < 4; ++blk)
        for (int tap = 0; tap < 9; ++tap)
            for (int o = 0; o < 32; ++o)
                for (int h = 0; h < 2; ++h) {
                    const int dy = tap / 3, dx = tap % 3;
                    std::memcpy(out + ((dy * 4 + blk) * 2 + h) * 1536 + (dx * 32 + o) * 16,
                                w2k + ((blk * 9 + tap) * 32 + o) * 32 + h * 16, 16);
                }
    return DN8_OK;
}

}  // extern "C"
