// conv1.cu -- dense-layer conv1 on sm_100a: BN+ReLU+u8 prologue, 1x1 INT8 GEMM on tcgen05
// (kind::i8, u8 x s8 -> s32 in TMEM), u8 requantisation epilogue into the bottleneck planes.
//
// GEMM: M = N*HW pixels (tiles of 128 rows), N = 128 bottleneck channels, K = c_in in groups of
// 32 channels (one store group = one MMA of K = 32). Persistent: one CTA per SM walks its tiles.
// Warp roles (17 warps):
//   warp 0       TMEM owner and MMA issuer (lane 0): per K group one
//                tcgen05.mma M128 N128 K32 into one of two TMEM accumulators (2 x 128 columns),
//                tcgen05.commit frees the stage; after the last group, the accumulator.
//   warps 1-8    prologue: 256 threads = 128 rows x 2 halves of 16 channels. Each stage: one
//                16-byte load of store bytes and one of weights (register-staged DEPTH stages
//                ahead, plus a bulk L2 prefetch PF stages ahead), the fp16 / fp32 prologue, and
//                16-byte stores into the 32B-swizzled K-major operand slots.
//   warps 9-16   epilogue: warp w reads TMEM lanes 32*(w%4).. (its 32 pixels) and 64 of the 128
//                columns, requantises to u8 and writes 16-byte rows into the planes [8][M][16].
#include "dn8_common.cuh"
#include "dn8_kernels.h"

namespace dn8 {

constexpr int C1_STAGES = 8;
constexpr int C1_DEPTH = 4;        // register-staged loads in flight per prologue thread
constexpr int C1_PF = 12;          // stages between the L2 prefetch and the consumption
constexpr int C1_WARPS = 17;
constexpr int C1_THREADS = 32 * C1_WARPS;
constexpr int C1_TILE_BYTES = 128 * 32;

size_t conv1_smem_bytes(int G) {
    return 2 * C1_STAGES * C1_TILE_BYTES + static_cast<size_t>(G) * 256 + 128 * 8 +
           8 * (2 * C1_STAGES + 4) + 16 + 1024;   // + alignment slack
}

template <bool F16>
__global__ void __launch_bounds__(C1_THREADS, 1) conv1_kernel(const dn8_conv1_args a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sA = smem;                                        // [S][128][32] swizzled
    uint8_t* sB = smem + C1_STAGES * C1_TILE_BYTES;            // [S][128][32] swizzled
    uint8_t* sTab = smem + 2 * C1_STAGES * C1_TILE_BYTES;      // prologue table, G * 256 bytes max
    float2* sGd = reinterpret_cast<float2*>(sTab + a.G * 256);
    uint64_t* full = reinterpret_cast<uint64_t*>(sGd + 128);
    uint64_t* empty = full + C1_STAGES;
    uint64_t* accf = empty + C1_STAGES;
    uint64_t* acce = accf + 2;
    uint32_t* s_tmem = reinterpret_cast<uint32_t*>(acce + 2);
    volatile int* s_abort = reinterpret_cast<volatile int*>(s_tmem + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int G = a.G, G0 = a.G0, HW = a.HW;
    const int rows = a.N * HW;
    const int ntiles = (rows + 127) / 128;
    const int my_tiles = static_cast<int>(blockIdx.x) < ntiles ? (ntiles - 1 - blockIdx.x) / gridDim.x + 1 : 0;
    const int T = my_tiles * G;

    if (threadIdx.x == 0) {
        for (int s = 0; s < C1_STAGES; ++s) {
            mbar_init(&full[s], 8);
            mbar_init(&empty[s], 1);
        }
        for (int k = 0; k < 2; ++k) {
            mbar_init(&accf[k], 1);
            mbar_init(&acce[k], 8);
        }
        *s_abort = 0;
        mbar_fence_init();
    }
    if (F16) {
        for (int i = threadIdx.x; i < G * 16; i += C1_THREADS)
            reinterpret_cast<uint2*>(sTab)[i] = reinterpret_cast<const uint2*>(a.ab)[i];
    } else {
        for (int i = threadIdx.x; i < G * 32; i += C1_THREADS)
            reinterpret_cast<float2*>(sTab)[i] = reinterpret_cast<const float2*>(a.ab)[i];
    }
    for (int i = threadIdx.x; i < 128; i += C1_THREADS) sGd[i] = reinterpret_cast<const float2*>(a.gd)[i];
    if (warp == 0) tmem_alloc(s_tmem, 256);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *s_tmem;

    if (warp == 0) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            const uint32_t idesc = idesc_u8s8(128, 128);
            const uint32_t a0 = smem_u32(sA), b0 = smem_u32(sB);
            int i = 0;
            for (int t = 0; t < my_tiles; ++t) {
                const int acc = t & 1;
                if (!mbar_wait(&acce[acc], ((t >> 1) & 1) ^ 1, a.err, s_abort, ERR_WAIT_ACC)) break;
                tc_fence_after();
                bool ok = true;
                for (int g = 0; g < G; ++g, ++i) {
                    const int s = i % C1_STAGES;
                    if (!mbar_wait(&full[s], (i / C1_STAGES) & 1, a.err, s_abort, ERR_WAIT_FULL)) { ok = false; break; }
                    tc_fence_after();
                    const uint64_t ad = sdesc(a0 + s * C1_TILE_BYTES, 16, 256, LAYOUT_SW32);
                    const uint64_t bd = sdesc(b0 + s * C1_TILE_BYTES, 16, 256, LAYOUT_SW32);
                    umma_u8s8(tmem + acc * 128, ad, bd, idesc, g > 0 ? 1u : 0u);
                    umma_commit(&empty[s]);
                }
                if (!ok) break;
                umma_commit(&accf[acc]);
            }
        }
        __syncwarp();
    } else if (warp <= 8) {
        // ---------------- prologue ----------------
        const int pt = threadIdx.x - 32;          // 0..255
        const int r = pt >> 1, h = pt & 1;
        const int swz = r * 32 + ((h ^ ((r >> 2) & 1)) << 4);
        const int8_t* wrow = a.w + static_cast<size_t>(r) * 32 + h * 16;
        // load position (stage i + DEPTH): tile index within this CTA, group, row pointers
        int ld_t = 0, ld_g = 0;
        const int8_t* ld_in0 = nullptr;           // row's in0 address (group 0), or null
        const int8_t* ld_seg = nullptr;           // row's seg address (layer group 0)
        auto set_tile = [&](int t) {
            const int m = (static_cast<int>(blockIdx.x) + t * static_cast<int>(gridDim.x)) * 128 + r;
            if (m < rows) {
                const int n = m / HW, p = m - n * HW;
                ld_in0 = a.in0 + (static_cast<size_t>(n) * G0 * HW + p) * 32 + h * 16;
                ld_seg = a.seg + static_cast<size_t>(m) * 32 + h * 16;
            } else {
                ld_in0 = ld_seg = nullptr;
            }
        };
        const size_t in0_g = static_cast<size_t>(HW) * 32, seg_g = static_cast<size_t>(rows) * 32;
        uint4 ra[C1_DEPTH], rb[C1_DEPTH];
        auto issue = [&](uint4& va, uint4& vb) {
            if (ld_in0 != nullptr) {
                const int8_t* src = ld_g < G0 ? ld_in0 + ld_g * in0_g : ld_seg + (ld_g - G0) * seg_g;
                va = __ldg(reinterpret_cast<const uint4*>(src));
            } else {
                va = make_uint4(0u, 0u, 0u, 0u);
            }
            vb = __ldg(reinterpret_cast<const uint4*>(wrow + static_cast<size_t>(ld_g) * 128 * 32));
            if (++ld_g == G) {
                ld_g = 0;
                if (++ld_t < my_tiles) set_tile(ld_t);
                else ld_in0 = ld_seg = nullptr;
            }
        };
        auto prefetch = [&](int i) {                // L2 prefetch of the A tile of stage i
            const int t = i / G, g = i - t * G;
            const int m0 = (static_cast<int>(blockIdx.x) + t * static_cast<int>(gridDim.x)) * 128;
            const int mrows = min(128, rows - m0);
            if (g >= G0) {
                prefetch_l2_bulk(a.seg + (static_cast<size_t>(g - G0) * rows + m0) * 32, mrows * 32);
            } else {
                int m = m0;
                while (m < m0 + mrows) {            // split at image boundaries
                    const int n = m / HW, p = m - n * HW;
                    const int cnt = min(m0 + mrows - m, HW - p);
                    prefetch_l2_bulk(a.in0 + ((static_cast<size_t>(n) * G0 + g) * HW + p) * 32, cnt * 32);
                    m += cnt;
                }
            }
        };
        if (my_tiles > 0) set_tile(0);
        if (pt == 0)
            for (int i = 0; i < C1_PF && i < T; ++i) prefetch(i);
#pragma unroll
        for (int k = 0; k < C1_DEPTH; ++k)
            if (k < T) issue(ra[k], rb[k]);
        int g = 0;
        for (int i0 = 0; i0 < T; i0 += C1_DEPTH) {
#pragma unroll
            for (int k = 0; k < C1_DEPTH; ++k) {
                const int i = i0 + k;
                if (i < T) {
                    const int s = i % C1_STAGES;
                    if (!mbar_wait(&empty[s], ((i / C1_STAGES) & 1) ^ 1, a.err, s_abort, ERR_WAIT_EMPTY)) {
                        i0 = T;
                        break;
                    }
                    if (pt == 0 && i + C1_PF < T) prefetch(i + C1_PF);
                    uint4 u;
                    if (F16) {
                        const uint2* tb = reinterpret_cast<const uint2*>(sTab) + g * 16 + h * 8;
                        const uint2 p0 = tb[0], p1 = tb[1], p2 = tb[2], p3 = tb[3];
                        const uint2 p4 = tb[4], p5 = tb[5], p6 = tb[6], p7 = tb[7];
                        u.x = prologue_f16x4(ra[k].x, p0.x, p0.y, p1.x, p1.y);
                        u.y = prologue_f16x4(ra[k].y, p2.x, p2.y, p3.x, p3.y);
                        u.z = prologue_f16x4(ra[k].z, p4.x, p4.y, p5.x, p5.y);
                        u.w = prologue_f16x4(ra[k].w, p6.x, p6.y, p7.x, p7.y);
                    } else {
                        const float2* tb = reinterpret_cast<const float2*>(sTab) + g * 32 + h * 16;
                        u.x = prologue_f32x4(ra[k].x, tb);
                        u.y = prologue_f32x4(ra[k].y, tb + 4);
                        u.z = prologue_f32x4(ra[k].z, tb + 8);
                        u.w = prologue_f32x4(ra[k].w, tb + 12);
                    }
                    *reinterpret_cast<uint4*>(sA + s * C1_TILE_BYTES + swz) = u;
                    *reinterpret_cast<uint4*>(sB + s * C1_TILE_BYTES + swz) = rb[k];
                    fence_async_smem();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&full[s]);
                    if (i + C1_DEPTH < T) issue(ra[k], rb[k]);
                    if (++g == G) g = 0;
                }
            }
        }
    } else {
        // ---------------- epilogue ----------------
        const int quad = warp & 3, chalf = (warp - 9) >> 2;
        uint8_t* out = a.out;
        for (int t = 0; t < my_tiles; ++t) {
            const int acc = t & 1;
            if (!mbar_wait(&accf[acc], (t >> 1) & 1, a.err, s_abort, ERR_WAIT_ACC)) break;
            tc_fence_after();
            const int m = (static_cast<int>(blockIdx.x) + t * static_cast<int>(gridDim.x)) * 128 + quad * 32 + lane;
            const uint32_t taddr = tmem + (static_cast<uint32_t>(quad * 32) << 16) + acc * 128 + chalf * 64;
#pragma unroll
            for (int half = 0; half < 2; ++half) {
                uint32_t v[32];
                tmem_ld32(taddr + half * 32, v);
                tmem_wait_ld();
                uint32_t wds[8];
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const int c = chalf * 64 + half * 32 + j * 4;
                    uint32_t wd = 0;
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        const float2 p = sGd[c + k];
                        wd |= epi_u8(static_cast<int32_t>(v[j * 4 + k]), p.x, p.y) << (8 * k);
                    }
                    wds[j] = wd;
                }
                if (m < rows) {
                    const int plane = chalf * 4 + half * 2;
                    *reinterpret_cast<uint4*>(out + (static_cast<size_t>(plane) * rows + m) * 16) =
                        make_uint4(wds[0], wds[1], wds[2], wds[3]);
                    *reinterpret_cast<uint4*>(out + (static_cast<size_t>(plane + 1) * rows + m) * 16) =
                        make_uint4(wds[4], wds[5], wds[6], wds[7]);
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acce[acc]);
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_free(tmem, 256);
    }
}

cudaError_t launch_conv1(const dn8_conv1_args& a, int sms, cudaStream_t st) {
    const int rows = a.N * a.HW;
    const int ntiles = (rows + 127) / 128;
    const int grid = ntiles < sms ? ntiles : sms;
    const size_t smem = conv1_smem_bytes(a.G);
    if (grid <= 0) return cudaSuccess;
    cudaError_t e;
    if (a.prologue_f16) {
        e = cudaFuncSetAttribute(conv1_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (e != cudaSuccess) return e;
        conv1_kernel<true><<<grid, C1_THREADS, smem, st>>>(a);
    } else {
        e = cudaFuncSetAttribute(conv1_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (e != cudaSuccess) return e;
        conv1_kernel<false><<<grid, C1_THREADS, smem, st>>>(a);
    }
    return cudaGetLastError();
}

}  // namespace dn8
