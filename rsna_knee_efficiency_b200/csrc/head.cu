// head.cu -- global pooling of the last block (norm5 with sigma folded, ReLU, spatial mean) and the
// linear head in one reduction kernel: a cluster of four CTAs per image, each pooling a quarter of
// the channel groups; the first CTA gathers the features over distributed shared memory.
//   features f[n][c] = (p0 + p1 + p2 + p3) / HW with p_q the fp32 sum, in ascending pixel order, of
//     relu(fmaf(a_c, q, b_c)) over pixels s = q, q + 4, ...: the reference's `final_q`
//     (src/knee/dense8s_kernels.cu:2306-2323), bit for bit;
//   logits l[n][j] = sum_c f[n][c] * Hw[j][c] + Hb[j] (fp32, fixed reduction order);
//   per view of V consecutive images the mean of the logits over the view (the slice mean), written
//   by the last CTA of the view to finish (an atomic ticket per view, reset for the next call).
#include <mutex>

#include "dn8_common.cuh"
#include "dn8_kernels.h"

namespace dn8 {

constexpr int HD_THREADS = 128;
constexpr int HD_CLUSTER = 4;              // CTAs per image: each pools a quarter of the groups
constexpr int HD_MAX_SLICE = 18;           // groups of a quarter (G <= 72, the 2304 channels dn8_head takes)

// Image n = blockIdx.x / HD_CLUSTER; CTA r of its cluster pools groups [r G / 4, (r + 1) G / 4).
// task = (group, 16-channel half, partial q): one 16-byte load per pixel feeds 16 channel sums; each
// channel's partial q is summed in ascending pixel order.
__global__ void __launch_bounds__(HD_THREADS, 1) head_kernel(const dn8_head_args a) {
    extern __shared__ float hs[];
    const int C = a.G * 32, HW = a.HW;
    const int n = blockIdx.x / HD_CLUSTER;
    const uint32_t rank = cluster_rank();
    const int g0 = static_cast<int>(rank) * a.G / HD_CLUSTER, g1 = (static_cast<int>(rank) + 1) * a.G / HD_CLUSTER;
    const size_t nal = static_cast<size_t>(a.n_alloc > a.N ? a.n_alloc : a.N);
    float* part = hs;                          // [4][HD_MAX_SLICE * 32]: this CTA's channels
    float* feat = hs + 4 * HD_MAX_SLICE * 32;  // [C] (this CTA's channels; rank 0 gathers all of them)
    float* red = feat + C;                     // [HD_THREADS / 32][NOUT]
    const int tid = threadIdx.x;
    griddep_launch_dependents();
    griddep_wait();                            // the last block's store
    constexpr int SL = HD_MAX_SLICE * 32;
    for (int task = tid; task < (g1 - g0) * 8; task += HD_THREADS) {
        const int g = g0 + (task >> 3), h = (task >> 2) & 1, q = task & 3;        // channels 16 h .. 16 h + 15
        // pixel s of image n in group g: group-major planes, or the tile-major store (pixel p = n HW + s
        // at tile p / 128, row p % 128)
        const int8_t* base;
        size_t tstride = 0, p0 = 0;
        // the tile-major store holds q + 128 per byte already (offset binary); planes hold signed q
        const uint32_t xm = a.tile_groups > 0 ? 0u : 0x80808080u;
        if (a.tile_groups > 0) {
            base = a.in0 + static_cast<size_t>(g) * 4096 + h * 16;
            tstride = static_cast<size_t>(a.tile_groups) << 12;
            p0 = static_cast<size_t>(n) * HW;
        } else {
            base = (g < a.G0 ? a.in0 + ((static_cast<size_t>(g) * nal + n) * HW) * 32
                             : a.seg + ((static_cast<size_t>(g - a.G0) * nal + n) * HW) * 32) + h * 16;
        }
        const float2* ab = reinterpret_cast<const float2*>(a.fab) + g * 32 + h * 16;
        float av[16], bv[16], acc[16];
#pragma unroll
        for (int k = 0; k < 16; ++k) {
            const float2 pr = ab[k];
            av[k] = pr.x;
            bv[k] = pr.y;
            acc[k] = 0.0f;
        }
        // (unrolled so that 16 pixels' loads are in flight: the chain of a thread is HW / 4 pixels long;
        // each channel's sum still runs in ascending pixel order)
#pragma unroll 16
        for (int s = q; s < HW; s += 4) {
            const size_t p = p0 + s;
            const int8_t* src = a.tile_groups > 0 ? base + (p >> 7) * tstride + (p & 127) * 32 : base + p * 32;
            const uint4 v = __ldg(reinterpret_cast<const uint4*>(src));
            const uint32_t w[4] = {v.x ^ xm, v.y ^ xm, v.z ^ xm, v.w ^ xm};
#pragma unroll
            for (int k = 0; k < 16; ++k) {
                // the byte q + 128 in the mantissa of 2^23: exact float q
                const float f = __int_as_float(__byte_perm(w[k >> 2], 0x4B000000u, 0x7540 | (k & 3))) - 8388736.0f;
                acc[k] += fmaxf(fmaf(av[k], f, bv[k]), 0.0f);
            }
        }
#pragma unroll
        for (int k = 0; k < 16; ++k) part[q * SL + (g - g0) * 32 + h * 16 + k] = acc[k];
    }
    __syncthreads();
    for (int c = g0 * 32 + tid; c < g1 * 32; c += HD_THREADS) {
        const int cl = c - g0 * 32;
        const float f = (part[cl] + part[SL + cl] + part[2 * SL + cl] + part[3 * SL + cl]) / static_cast<float>(HW);
        feat[c] = f;
        if (a.feat != nullptr) a.feat[static_cast<size_t>(n) * C + c] = f;
    }
    cluster_sync();                            // every CTA's features are in its shared memory
    if (rank == 0 && a.hw != nullptr) {
        // gather the other CTAs' channels (distributed shared memory)
        for (uint32_t r = 1; r < HD_CLUSTER; ++r) {
            const int c0 = static_cast<int>(r) * a.G / HD_CLUSTER * 32, c1 = (static_cast<int>(r) + 1) * a.G / HD_CLUSTER * 32;
            for (int c = c0 + tid; c < c1; c += HD_THREADS) feat[c] = ld_peer_f32(&feat[c], r);
        }
    }
    cluster_sync();                            // the peers' shared memory stays until rank 0 has read it
    if (rank != 0 || a.hw == nullptr) return;
    __syncthreads();
    // logits: each warp reduces a strided share of the channels for every output, then a fixed tree
    const int warp = tid >> 5, lane = tid & 31, nw = HD_THREADS / 32;
    for (int j = 0; j < a.n_out; ++j) {
        float sm = 0.0f;
        for (int c = tid; c < C; c += HD_THREADS) sm = fmaf(feat[c], a.hw[static_cast<size_t>(j) * C + c], sm);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sm += __shfl_xor_sync(0xffffffffu, sm, o);
        if (lane == 0) red[warp * a.n_out + j] = sm;
    }
    __syncthreads();
    if (tid < a.n_out) {
        float sm = 0.0f;
        for (int w = 0; w < nw; ++w) sm += red[w * a.n_out + tid];
        a.logits[static_cast<size_t>(n) * a.n_out + tid] = sm + a.hb[tid];
    }
    if (a.view_logits == nullptr || a.per_view < 1) return;
    // the last image of a view to finish averages the view's logits in image order
    __shared__ int s_last;
    __threadfence();
    __syncthreads();
    const int v = n / a.per_view;
    if (tid == 0) {
        const int ticket = atomicAdd(a.tickets + v, 1);
        s_last = ticket == a.per_view - 1;
    }
    __syncthreads();
    if (s_last) {
        __threadfence();
        if (tid < a.n_out) {
            float sm = 0.0f;
            for (int k = 0; k < a.per_view; ++k)
                sm += __ldcg(a.logits + static_cast<size_t>(v * a.per_view + k) * a.n_out + tid);
            a.view_logits[static_cast<size_t>(v) * a.n_out + tid] = sm / static_cast<float>(a.per_view);
        }
        if (tid == 0) a.tickets[v] = 0;
    }
}

// Built-in ticket scratch of dn8_head_noalloc: one counter per view, zero at module load and left
// zero by every completed call (the last image of a view resets its counter).
static __device__ __align__(256) int32_t g_view_tickets[DN8_HEAD_SCRATCH_VIEWS];

namespace {
std::mutex g_scratch_mu;
int32_t* g_scratch_ptr[DN8_MAX_DEVICES] = {};
}  // namespace

// Device address of the current device's ticket scratch, looked up once per device (the first
// call can load the module on that device, so it should not happen inside stream capture).
cudaError_t head_scratch_tickets(int32_t** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= DN8_MAX_DEVICES) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    if (g_scratch_ptr[dev] == nullptr) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_view_tickets);
        if (e != cudaSuccess) return e;
        g_scratch_ptr[dev] = static_cast<int32_t*>(p);
    }
    *out = g_scratch_ptr[dev];
    return cudaSuccess;
}

cudaError_t launch_head(const dn8_head_args& a, cudaStream_t st, bool pdl) {
    const int C = a.G * 32;
    const size_t smem =
        (static_cast<size_t>(4) * HD_MAX_SLICE * 32 + C + (HD_THREADS / 32) * (a.n_out > 0 ? a.n_out : 1)) * sizeof(float);
    if (a.G > HD_CLUSTER * HD_MAX_SLICE) return cudaErrorInvalidValue;
    cudaError_t e = cudaFuncSetAttribute(head_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    return launch_pdl_cluster(pdl, HD_CLUSTER, head_kernel, dim3(a.N * HD_CLUSTER), dim3(HD_THREADS), smem, st, a);
}

}  // namespace dn8
