// conv2.cu -- dense-layer conv2 on sm_100a: 3x3 pad-1 conv 128 -> 32 on the u8 bottleneck,
// int8 requantisation straight into the block store slot (the layer's [N][HW][32] segment, or its
// group of a tile-major block store: pixel p at tile p / 128, row p % 128).
//
// Formulation ("dx in N"): a tile is Rt = 128 / W full image rows (128 pixels, W <= 128). For
// each kernel row dy and channel block c (12 K steps of 32 channels) one
// tcgen05.mma M128 N96 K32 multiplies the tile's pixels shifted by dy rows (A: a shifted view of
// the bottleneck rows held in shared memory, no copy) by the weights of the three taps dx of
// that row stacked along N (96 = 3 dx x 32 outputs):
//     D[p][dx, o] = sum_{dy, c} W[dy, dx][o][c] * X[y(p) + dy - 1, x(p)][c].
// The epilogue adds the three column taps: out[p][o] = D[p-1][0, o] + D[p][1, o] + D[p+1][2, o]
// (neighbours through warp shuffles, zero outside the row), so no column halo is ever loaded.
// One 4-D TMA load per tile brings the 8 bottleneck planes x (Rt + 2) image rows; rows outside
// the image arrive zero-filled (the convolution's zero padding). The weights arrive prepared
// (dn8_prepare_conv2_weights) in one bulk copy and stay resident.
// Warp roles: warp 0 TMEM owner + TMA producer, warp 1 MMA issuer, warps 2-17 epilogue in two
// groups of 8 that take alternate tiles (group g: tiles t = g, g + 2, ..., accumulator g), so two
// tiles are requantised at once; warp w reads TMEM lanes 32*(w%4).. and 16 of the 32 outputs.
#include "dn8_common.cuh"
#include "dn8_kernels.h"

namespace dn8 {

// Input ring depth: 5 stages where they fit (maps up to 64 x 64: a tile's MMAs are short there, so
// the loads have to run further ahead; -6 % at 32 x 32), else 3 (128 x 128: 48 KB stages). A
// compile-time depth per kernel instance keeps the ring arithmetic constant.
constexpr int C2_STAGES_DEEP = 5, C2_STAGES = 3;
constexpr int C2_THREADS = 576;
constexpr int C2_W_BYTES = 36864;            // [dy][cblk][2 halves][96 rows][16 B]
constexpr int C2_XBUF = 4;                   // edge-exchange buffers (tile t uses t % 4: one group's)

static inline int c2_rows_per_tile(int H, int W) {
    int rt = 128 / W;
    return rt < H ? rt : H;
}
// A stage holds 8 planes of (Rt + 2) rows; the MMA of the last plane reads 128 rows from row 2,
// which can run past the plane when Rt * W < 128 (junk rows): the stage is sized to cover it.
static inline size_t c2_stage_bytes(int Rt, int W) {
    const size_t pl = static_cast<size_t>(Rt + 2) * W * 16;
    const size_t need = 7 * pl + static_cast<size_t>(2 * W + 128) * 16;
    const size_t b = need > 8 * pl ? need : 8 * pl;
    return ((b + 1023) / 1024) * 1024;
}
static inline size_t c2_smem_for(int ns, size_t stage) {
    return 1024 + C2_W_BYTES + ns * stage + 128 + C2_XBUF * 2 * 4 * 2 * 16 * 4 + 8 * (2 * ns + 5 + 2 * C2_XBUF) + 16;
}
static inline int c2_stages(int H, int W) {
    return c2_smem_for(C2_STAGES_DEEP, c2_stage_bytes(c2_rows_per_tile(H, W), W)) <= 227 * 1024 ? C2_STAGES_DEEP
                                                                                                  : C2_STAGES;
}
size_t conv2_smem_bytes(int H, int W) {
    return c2_smem_for(c2_stages(H, W), c2_stage_bytes(c2_rows_per_tile(H, W), W));
}

template <int NS>
__global__ void __launch_bounds__(C2_THREADS, 1)
conv2_kernel(const __grid_constant__ CUtensorMap tmap, const dn8_conv2_args a, int Rt, uint32_t stage_bytes) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sW = smem;
    uint8_t* sX = smem + C2_W_BYTES;                       // stages, 1024-aligned (36864 = 36 * 1024)
    float* sSc = reinterpret_cast<float*>(sX + NS * stage_bytes);
    int32_t* xb = reinterpret_cast<int32_t*>(sSc + 32);    // [XBUF][2 ch][4 quad][2][16]
    uint64_t* full = reinterpret_cast<uint64_t*>(xb + C2_XBUF * 2 * 4 * 2 * 16);
    uint64_t* empty = full + NS;
    uint64_t* accf = empty + NS;
    uint64_t* acce = accf + 2;
    uint64_t* xbar = acce + 2;                             // [XBUF][2 ch]: neighbour exchange
    uint64_t* wfull = xbar + 2 * C2_XBUF;
    uint32_t* s_tmem = reinterpret_cast<uint32_t*>(wfull + 1);
    volatile int* s_abort = reinterpret_cast<volatile int*>(s_tmem + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int H = a.H, W = a.W;
    const int tpi = (H + Rt - 1) / Rt;
    const int ntiles = a.N * tpi;
    const int my_tiles = static_cast<int>(blockIdx.x) < ntiles ? (ntiles - 1 - blockIdx.x) / gridDim.x + 1 : 0;
    const uint32_t PL = static_cast<uint32_t>((Rt + 2) * W * 16);     // one plane of a stage

    if (threadIdx.x == 0) {
        for (int s = 0; s < NS; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int k = 0; k < 2; ++k) {
            mbar_init(&accf[k], 1);
            mbar_init(&acce[k], 8);
        }
        for (int k = 0; k < 2 * C2_XBUF; ++k) mbar_init(&xbar[k], 4);
        mbar_init(&wfull[0], 1);
        *s_abort = 0;
        mbar_fence_init();
        prefetch_tensormap(&tmap);
    }
    // exact int32 -> float through the magic add when every channel saturates at +-2^22 (see gemm.cu)
    int ok = 1;
    if (threadIdx.x < 32) {
        const float sc = a.sc[threadIdx.x];
        sSc[threadIdx.x] = sc;
        ok = sc * 4194304.0f >= 127.0f ? 1 : 0;
    }
    if (warp == 0) tmem_alloc(s_tmem, 256);
    tc_fence_before();
    const int fast_cvt = __syncthreads_and(ok);
    tc_fence_after();
    const uint32_t tmem = *s_tmem;
    if (threadIdx.x == 0 && my_tiles > 0) {
        // the prepared weights [dy][cblk][half][dx * 32 + o][16] in one bulk copy (constant: it
        // may land while the previous kernel still runs)
        mbar_expect_tx(&wfull[0], C2_W_BYTES);
        bulk_g2s(sW, a.w, C2_W_BYTES, &wfull[0]);
    }
    griddep_launch_dependents();
    griddep_wait();                                    // the bottleneck of this layer's conv1

    if (warp == 0) {
        // ---------------- TMA producer ----------------
        if (lane == 0 && my_tiles > 0) {
            for (int t = 0; t < my_tiles; ++t) {
                const int s = t % NS;
                if (!mbar_wait(&empty[s], ((t / NS) & 1) ^ 1, a.err, s_abort, ERR_WAIT_EMPTY | (33 << 4))) break;
                const int tile = blockIdx.x + t * gridDim.x;
                const int n = tile / tpi, y0 = (tile - n * tpi) * Rt;
                mbar_expect_tx(&full[s], 8u * PL);
                tma_load_4d(sX + s * stage_bytes, &tmap, &full[s], 0, y0 - 1, n, 0);
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        // ---------------- MMA issuer (the whole warp; one elected lane issues) ----------------
        const uint32_t idesc = idesc_u8s8(128, 96);
        const uint32_t x0 = smem_u32(sX), w0 = smem_u32(sW);
        const bool wok = my_tiles == 0 || mbar_wait_w(&wfull[0], 0, a.err, s_abort, ERR_WAIT_FULL | (34 << 4));
        for (int t = 0; t < my_tiles && wok; ++t) {
            const int acc = t & 1, s = t % NS;
            if (!mbar_wait_w(&acce[acc], ((t >> 1) & 1) ^ 1, a.err, s_abort, ERR_WAIT_ACC | (35 << 4))) break;
            tc_fence_after();
            if (!mbar_wait_w(&full[s], (t / NS) & 1, a.err, s_abort, ERR_WAIT_FULL | (36 << 4))) break;
            tc_fence_after();
            const uint32_t xs = x0 + s * stage_bytes;
#pragma unroll
            for (int dy = 0; dy < 3; ++dy)
#pragma unroll
                for (int cb = 0; cb < 4; ++cb) {
                    const uint64_t ad = sdesc(xs + 2 * cb * PL + dy * W * 16, PL, 128, LAYOUT_NONE);
                    const uint64_t bd = sdesc(w0 + (dy * 4 + cb) * 3072, 1536, 128, LAYOUT_NONE);
                    umma_u8s8_w(tmem + acc * 128, ad, bd, idesc, (dy | cb) ? 1u : 0u);
                }
            umma_commit_w(&empty[s]);
            umma_commit_w(&accf[acc]);
        }
        __syncwarp();
    } else {
        // ---------------- epilogue ----------------
        // Group g = (warp - 2) / 8 takes tiles g, g + 2, ... (accumulator g). Per tile: load the
        // accumulator (releasing it to the MMA at once), publish the edge columns, wait for the
        // other three quads' edges (exchange t), finish. Tile t's edges live in buffer t % 4, whose
        // previous user is tile t - 4 of the same group: before writing it, a warp has waited for
        // exchange t - 2, by which every warp of its channel half and group has finished tile t - 4.
        const int quad = warp & 3, ch = ((warp - 2) >> 2) & 1, grp = (warp - 2) >> 3;
        const int p = quad * 32 + lane;                       // pixel within the tile
        const int yl = p / W, x = p - yl * W;
        const bool has_l = x > 0, has_r = x < W - 1;
        const bool at_l = lane == 0, at_r = lane == 31;
        const float4* sc4 = reinterpret_cast<const float4*>(sSc + ch * 16);   // this half's output scales
        const int ql = quad > 0 ? quad - 1 : 0, qr = quad < 3 ? quad + 1 : 3;

        auto load = [&](int t, uint32_t (&d0)[16], uint32_t (&d1)[16], uint32_t (&d2)[16]) -> bool {
            const int acc = t & 1;
            if (!mbar_wait(&accf[acc], (t >> 1) & 1, a.err, s_abort, ERR_WAIT_ACC | (37 << 4))) return false;
            tc_fence_after();
            const uint32_t taddr = tmem + (static_cast<uint32_t>(quad * 32) << 16) + acc * 128 + ch * 16;
            tmem_ld16(taddr, d0);
            tmem_ld16(taddr + 32, d1);
            tmem_ld16(taddr + 64, d2);
            tmem_wait_ld(d0);
            reg_bind(d1);
            reg_bind(d2);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acce[acc]);
            return true;
        };
        auto publish = [&](int t, const uint32_t (&d0)[16], const uint32_t (&d2)[16]) {
            // lane 31's left tap D[p][0] and lane 0's right tap D[p][2] for the neighbour quads
            int32_t* xq = xb + ((t % C2_XBUF) * 2 + ch) * 4 * 32;      // [quad][2][16]
            if (at_r)
#pragma unroll
                for (int j = 0; j < 4; ++j)
                    *reinterpret_cast<uint4*>(xq + quad * 32 + 4 * j) =
                        make_uint4(d0[4 * j], d0[4 * j + 1], d0[4 * j + 2], d0[4 * j + 3]);
            if (at_l)
#pragma unroll
                for (int j = 0; j < 4; ++j)
                    *reinterpret_cast<uint4*>(xq + quad * 32 + 16 + 4 * j) =
                        make_uint4(d2[4 * j], d2[4 * j + 1], d2[4 * j + 2], d2[4 * j + 3]);
            __syncwarp();
            if (lane == 0) mbar_arrive(&xbar[(t % C2_XBUF) * 2 + ch]);
        };
        auto wait_x = [&](int t) -> bool {
            return mbar_wait(&xbar[(t % C2_XBUF) * 2 + ch], (t / C2_XBUF) & 1, a.err, s_abort, ERR_WAIT_ACC | (38 << 4));
        };
        // out[p] = D[p-1][0] + D[p][1] + D[p+1][2] (zero outside the row). The in-warp neighbours are
        // added right after the load (so 16 sums, not 48 taps, stay live across the exchange);
        // lanes 0 and 31 add the other quads' edge taps once exchange t is done.
        auto fold = [&](const uint32_t (&d0)[16], const uint32_t (&d1)[16], const uint32_t (&d2)[16],
                        int32_t (&sum)[16]) {
            const bool in_l = has_l && !at_l, in_r = has_r && !at_r;
#pragma unroll
            for (int o = 0; o < 16; ++o) {
                const uint32_t l = __shfl_up_sync(0xffffffffu, d0[o], 1);
                const uint32_t r = __shfl_down_sync(0xffffffffu, d2[o], 1);
                sum[o] = static_cast<int32_t>(d1[o]) + (in_l ? static_cast<int32_t>(l) : 0) +
                         (in_r ? static_cast<int32_t>(r) : 0);
            }
        };
        // the rounding add whose low byte is q (1.5 * 2^23), or q + 128 into a tile-major store
        // (offset binary; the sum stays even, so ties still round to even q)
        const float omag = a.tile_groups > 0 ? 12583040.0f : 12582912.0f;
        auto finish = [&](int t, const int32_t (&sum)[16]) {
            const int32_t* xq = xb + ((t % C2_XBUF) * 2 + ch) * 4 * 32;
            const bool ex_l = has_l && at_l, ex_r = has_r && at_r;
            uint32_t wd[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                // the other quads' edge taps count only for lanes 0 / 31 inside the image row: the
                // other lanes read nothing and add zero
                uint4 el = make_uint4(0u, 0u, 0u, 0u), er = make_uint4(0u, 0u, 0u, 0u);
                if (ex_l) el = *reinterpret_cast<const uint4*>(xq + ql * 32 + 4 * j);
                if (ex_r) er = *reinterpret_cast<const uint4*>(xq + qr * 32 + 16 + 4 * j);
                const uint32_t le[4] = {el.x, el.y, el.z, el.w};
                const uint32_t re[4] = {er.x, er.y, er.z, er.w};
                const float4 s4 = sc4[j];                             // broadcast read, 4 scales
                const float sc[4] = {s4.x, s4.y, s4.z, s4.w};
                uint32_t q[4];
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const int32_t accv = sum[4 * j + k] + static_cast<int32_t>(le[k]) + static_cast<int32_t>(re[k]);
                    const float f = fast_cvt ? __int_as_float(accv + 0x4B400000) - 12582912.0f
                                             : __int2float_rn(accv);
                    // rint(clamp(f sc, +-127)) (+ 128) as the low byte of (clamped + omag)
                    q[k] = __float_as_uint(fminf(fmaxf(f * sc[k], -127.0f), 127.0f) + omag);
                }
                wd[j] = __byte_perm(__byte_perm(q[0], q[1], 0x0040), __byte_perm(q[2], q[3], 0x0040), 0x5410);
            }
            const int tile = blockIdx.x + t * gridDim.x;
            const int n = tile / tpi, y0 = (tile - n * tpi) * Rt;
            if (yl < Rt && y0 + yl < H) {
                // pixel p of the slot [N][H*W][32], or group `group` of the tile-major block store
                const size_t px = (static_cast<size_t>(n) * H + y0 + yl) * W + x;
                int8_t* dst = a.tile_groups > 0
                                  ? a.out + (((px >> 7) * a.tile_groups + a.group) << 12) + (px & 127) * 32 + ch * 16
                                  : a.out + px * 32 + ch * 16;
                *reinterpret_cast<uint4*>(dst) = make_uint4(wd[0], wd[1], wd[2], wd[3]);
            }
        };
        for (int t = grp; t < my_tiles; t += 2) {
            int32_t sum[16];
            {
                uint32_t d0[16], d1[16], d2[16];
                if (!load(t, d0, d1, d2)) break;
                publish(t, d0, d2);
                fold(d0, d1, d2, sum);
            }
            if (!wait_x(t)) break;
            finish(t, sum);
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_free(tmem, 256);
    }
}

// 4-D map over the bottleneck planes [8][N][H][W * 16 bytes] with 8-byte elements, so that a box
// row is a whole image row (16 W bytes; TMA moves long rows far faster than 16-byte ones):
// box {2W, Rt + 2, 1, 8}; rows outside [0, H) are zero-filled.
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static cudaError_t make_bott_map(CUtensorMap* map, const void* base, int N, int H, int W, int Rt) {
    static EncodeTiledFn encode = nullptr;
    if (encode == nullptr) {
        cudaDriverEntryPointQueryResult q;
        void* fn = nullptr;
        cudaError_t e = cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000,
                                                         cudaEnableDefault, &q);
        if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || fn == nullptr) return cudaErrorNotSupported;
        encode = reinterpret_cast<EncodeTiledFn>(fn);
    }
    const cuuint64_t rows = static_cast<cuuint64_t>(N) * H * W;
    cuuint64_t dims[4] = {2 * static_cast<cuuint64_t>(W), static_cast<cuuint64_t>(H), static_cast<cuuint64_t>(N), 8};
    cuuint64_t strides[3] = {static_cast<cuuint64_t>(W) * 16, static_cast<cuuint64_t>(H) * W * 16, rows * 16};
    cuuint32_t box[4] = {2 * static_cast<cuuint32_t>(W), static_cast<cuuint32_t>(Rt + 2), 1, 8};
    cuuint32_t estr[4] = {1, 1, 1, 1};
    CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT64, 4, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

cudaError_t prepare_conv2(Conv2Plan* plan, const dn8_conv2_args& a) {
    if (a.W < 1 || a.W > 128 || a.H < 1 || a.N < 1) return cudaErrorInvalidValue;
    plan->Rt = c2_rows_per_tile(a.H, a.W);
    plan->stage_bytes = static_cast<uint32_t>(c2_stage_bytes(plan->Rt, a.W));
    plan->smem = conv2_smem_bytes(a.H, a.W);
    if (plan->smem > 227 * 1024) return cudaErrorInvalidValue;
    return make_bott_map(&plan->map, a.x, a.N, a.H, a.W, plan->Rt);
}

cudaError_t launch_conv2(const Conv2Plan& plan, const dn8_conv2_args& a, int sms, cudaStream_t st, bool pdl) {
    const int tpi = (a.H + plan.Rt - 1) / plan.Rt;
    const int ntiles = a.N * tpi;
    const int grid = ntiles < sms ? ntiles : sms;
    if (grid <= 0) return cudaSuccess;
    const auto kernel = c2_stages(a.H, a.W) == C2_STAGES_DEEP ? conv2_kernel<C2_STAGES_DEEP> : conv2_kernel<C2_STAGES>;
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(plan.smem));
    if (e != cudaSuccess) return e;
    return launch_pdl(pdl, kernel, dim3(grid), dim3(C2_THREADS), plan.smem, st, plan.map, a, plan.Rt,
                      plan.stage_bytes);
}

}  // namespace dn8
