// stem.cu -- the INT8 stem on sm_100a, fused with the input producer: pixels -> u8 (the uint8
// volume planes directly, or rint(255 sat(x)) of fp16 windows), optional horizontal flip, 7x7/2
// pad-3 conv 3 -> 64 on tcgen05 (kind::i8), q = rint(clamp(fmaf(acc, k, c), 0, 127)), 3x3/2 pad-1
// max-pool on the bytes, into block 1's group-major input [2][N][H/4 * W/4][32].
// Arithmetic of the reference's `stem_i8_body` (src/knee/dense8s_kernels.cu:3641-3771) and
// `stem_q_i8` (src/knee/dense8s.py:625-643).
//
// K layout (the reference's `stem_weights8`, dense8s.py:532-541): k = (ch * 7 + ky) * 8 + kx',
// kx' = kx + 1 (kx' = 0 has zero weight): 21 slots of 8 bytes; slot (ch, ky) of conv pixel cx is the
// 8 input bytes of row 2 cy + ky - 3 starting at column 2 cx - 4. K is padded to 192 (6 MMA steps).
//
// A CTA walks bands of BP pooled rows of one image; for every conv row of the band (2 BP + 1, the
// first one is the halo shared with the band above):
//   warps 1-4  load the two new input rows (all 3 channels) into a 16-row ring (column c at byte
//              c + 4, four zero bytes either side), build the im2col tile of the conv row
//              (ceil(CW / 128) M-tiles x 6 K steps, 32B-swizzled), double-buffered;
//   warp 0     TMEM owner / MMA issuer: M128 N64 K32 MMAs into one of two TMEM accumulators;
//   warps 5-8  requantise into a 3-row ring of conv outputs; after every odd conv row 2 py + 1 they
//              max-pool pooled row py (conv rows 2py-1 .. 2py+1) and write it out.
#include "dn8_common.cuh"
#include "dn8_kernels.h"

namespace dn8 {

constexpr int ST_THREADS = 288;
constexpr int ST_BP = 16;                 // pooled rows per band
constexpr int ST_RING = 16;               // input row ring
constexpr int ST_KSTEPS = 6;
constexpr int ST_WBYTES = ST_KSTEPS * 64 * 32;   // prepared weights [6][64][32] swizzled

struct StemGeo {
    int N, H, W;                           // input
    int CH, CW, PH, PW;                    // conv / pooled output
    int mt;                                // M-tiles per conv row
    int row_bytes;                         // one ring row of one channel: W + 8
    size_t ring_off, a_off, conv_off, bar_off, smem;
};

static StemGeo stem_geo(int N, int H, int W) {
    StemGeo g{};
    g.N = N; g.H = H; g.W = W;
    g.CH = H / 2; g.CW = W / 2; g.PH = H / 4; g.PW = W / 4;
    g.mt = (g.CW + 127) / 128;
    g.row_bytes = ((W + 12 + 15) / 16) * 16;        // the last slot reads up to byte W + 10
    size_t off = ST_WBYTES;                                               // weights at 0
    g.ring_off = off; off += static_cast<size_t>(ST_RING) * 3 * g.row_bytes;
    off = (off + 1023) / 1024 * 1024;
    g.a_off = off; off += static_cast<size_t>(2) * g.mt * ST_KSTEPS * 4096;   // 2 buffers
    g.conv_off = off; off += static_cast<size_t>(3) * g.mt * 128 * 64;        // 3 conv rows
    g.bar_off = off; off += 256 + 1024;                                       // kc, barriers
    g.smem = off + 1024;
    return g;
}

__global__ void __launch_bounds__(ST_THREADS, 1)
stem_kernel(const dn8_stem_args a, const StemGeo geo) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sW = smem;
    uint8_t* sRing = smem + geo.ring_off;
    uint8_t* sA = smem + geo.a_off;
    uint8_t* sC = smem + geo.conv_off;
    float* sKC = reinterpret_cast<float*>(smem + geo.bar_off);               // [128] k, c
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + geo.bar_off + 512);
    uint64_t* fullA = bars;          // [2] im2col tile ready (4 producer warps)
    uint64_t* emptyA = bars + 2;     // [2] MMA done with the tile
    uint64_t* accf = bars + 4;       // [2]
    uint64_t* acce = bars + 6;       // [2] (4 epilogue warps)
    uint64_t* wfull = bars + 8;      // weights landed
    uint64_t* ringrdy = bars + 9;    // [2] input rows of conv row i loaded (4 producer warps)
    uint64_t* written = bars + 11;   // [2] conv row i in the conv ring (4 epilogue warps)
    uint64_t* done = bars + 13;      // [2] conv row i finished, pooling included (4 epilogue warps)
    uint32_t* s_tmem = reinterpret_cast<uint32_t*>(bars + 16);
    volatile int* s_abort = reinterpret_cast<volatile int*>(s_tmem + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int H = geo.H, W = geo.W, CH = geo.CH, CW = geo.CW, PH = geo.PH, PW = geo.PW, MT = geo.mt;
    const int RB = geo.row_bytes;
    const int bands = (PH + ST_BP - 1) / ST_BP;
    const int ntask = geo.N * bands;
    const int my_tasks = static_cast<int>(blockIdx.x) < ntask ? (ntask - 1 - blockIdx.x) / gridDim.x + 1 : 0;

    if (threadIdx.x == 0) {
        for (int k = 0; k < 2; ++k) {
            mbar_init(&fullA[k], 4);
            mbar_init(&emptyA[k], 1);
            mbar_init(&accf[k], 1);
            mbar_init(&acce[k], 4);
            mbar_init(&ringrdy[k], 4);
            mbar_init(&written[k], 4);
            mbar_init(&done[k], 4);
        }
        mbar_init(&wfull[0], 1);
        *s_abort = 0;
        mbar_fence_init();
    }
    // k, c and the fast-conversion check (saturation beyond +-2^22, see gemm.cu)
    int ok = 1;
    if (threadIdx.x < 64) {
        const float k = a.kc[threadIdx.x], c = a.kc[64 + threadIdx.x];
        sKC[threadIdx.x] = k;
        sKC[64 + threadIdx.x] = c;
        ok = (fmaf(4194304.0f, k, c) >= 127.0f && fmaf(-4194304.0f, k, c) <= 0.0f) ? 1 : 0;
    }
    // zero the ring (its pad columns stay zero: row loads only write columns 0 .. W-1)
    for (int i = threadIdx.x; i < ST_RING * 3 * RB / 16; i += ST_THREADS)
        reinterpret_cast<uint4*>(sRing)[i] = make_uint4(0u, 0u, 0u, 0u);
    if (warp == 0) tmem_alloc(s_tmem, 256);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *s_tmem;
    if (warp >= 5) {                                      // arm both accumulators with MAGIC
        uint32_t arm[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) arm[j] = ACC_MAGIC;
        const int quad = warp & 3;
        for (int acc = 0; acc < 2; ++acc)
            for (int m = 0; m < MT; ++m)
                for (int cb = 0; cb < 64; cb += 32)
                    tmem_st32(tmem + (static_cast<uint32_t>(quad * 32) << 16) + acc * 128 + m * 64 + cb, arm);
        tmem_wait_st();
    }
    tc_fence_before();
    const int fast_cvt = __syncthreads_and(ok);
    tc_fence_after();

    // conv rows of task t: band b of image n -> conv rows cr0 .. cr0 + nrows - 1
    auto task_rows = [&](int t, int& n, int& py0, int& cr0, int& nrows) {
        const int task = blockIdx.x + t * gridDim.x;
        n = task / bands;
        const int b = task - n * bands;
        py0 = b * ST_BP;
        const int py1 = min(PH, py0 + ST_BP);
        cr0 = max(0, 2 * py0 - 1);
        nrows = min(CH - 1, 2 * py1 - 1) - cr0 + 1;
    };

    if (warp == 0) {
        // ---------------- MMA issuer ----------------
        if (lane == 0 && my_tasks > 0) {
            mbar_expect_tx(&wfull[0], ST_WBYTES);
            bulk_g2s(sW, a.w, ST_WBYTES, &wfull[0]);
            bool ok_run = mbar_wait(&wfull[0], 0, a.err, s_abort, ERR_WAIT_FULL);
            const uint32_t idesc = idesc_u8s8(128, 64);
            const uint32_t a0 = smem_u32(sA), w0 = smem_u32(sW);
            int i = 0;
            for (int t = 0; t < my_tasks && ok_run; ++t) {
                int n, py0, cr0, nrows;
                task_rows(t, n, py0, cr0, nrows);
                for (int r = 0; r < nrows; ++r, ++i) {
                    const int b = i & 1;
                    if (!mbar_wait(&acce[b], ((i >> 1) & 1) ^ 1, a.err, s_abort, ERR_WAIT_ACC)) { ok_run = false; break; }
                    if (!mbar_wait(&fullA[b], (i >> 1) & 1, a.err, s_abort, ERR_WAIT_FULL)) { ok_run = false; break; }
                    tc_fence_after();
                    for (int m = 0; m < MT; ++m)
#pragma unroll
                        for (int kk = 0; kk < ST_KSTEPS; ++kk) {
                            const uint64_t ad = sdesc(a0 + ((b * MT + m) * ST_KSTEPS + kk) * 4096, 16, 256, LAYOUT_SW32);
                            const uint64_t bd = sdesc(w0 + kk * 2048, 16, 256, LAYOUT_SW32);
                            umma_u8s8(tmem + b * 128 + m * 64, ad, bd, idesc, 1u);
                        }
                    umma_commit(&emptyA[b]);
                    umma_commit(&accf[b]);
                }
            }
        }
        __syncwarp();
    } else if (warp <= 4) {
        // ---------------- input rows + im2col ----------------
        const int pt = threadIdx.x - 32;                  // 0..127
        // load input row y (all 3 channels) of image n into ring slot y % ST_RING
        auto load_row = [&](int n, int y) {
            uint8_t* dst = sRing + (y & (ST_RING - 1)) * 3 * RB;
            const bool inside = y >= 0 && y < H;
            const int flip = a.flags != nullptr ? (a.flags[n] & 1) : 0;
            for (int ch = 0; ch < 3; ++ch) {
                uint8_t* drow = dst + ch * RB + 4;
                if (a.x_u8) {
                    const uint8_t* src = nullptr;
                    if (inside) {
                        const int plane = a.src[n * 4 + ch];
                        src = static_cast<const uint8_t*>(a.x) + (static_cast<size_t>(plane) * H + y) * W;
                    }
                    for (int c4 = pt; c4 < W / 4; c4 += 128) {
                        uint32_t v = inside ? __ldg(reinterpret_cast<const uint32_t*>(src) + c4) : 0u;
                        int col = 4 * c4;
                        if (flip) {
                            v = __byte_perm(v, 0, 0x0123);
                            col = W - 4 - col;
                        }
                        *reinterpret_cast<uint32_t*>(drow + col) = v;
                    }
                } else {
                    const uint16_t* src = inside ? static_cast<const uint16_t*>(a.x) + ((static_cast<size_t>(n) * 3 + ch) * H + y) * W
                                                 : nullptr;
                    for (int c4 = pt; c4 < W / 4; c4 += 128) {
                        uint32_t v = 0u;
                        if (inside) {
                            const uint2 hv = __ldg(reinterpret_cast<const uint2*>(src) + c4);
                            v = u8_of_f16x2(hv.x) | (u8_of_f16x2(hv.y) << 16);
                        }
                        int col = 4 * c4;
                        if (flip) {
                            v = __byte_perm(v, 0, 0x0123);
                            col = W - 4 - col;
                        }
                        *reinterpret_cast<uint32_t*>(drow + col) = v;
                    }
                }
            }
        };
        int i = 0;
        for (int t = 0; t < my_tasks; ++t) {
            int n, py0, cr0, nrows;
            task_rows(t, n, py0, cr0, nrows);
            bool ok_run = true;
            for (int r = 0; r < nrows; ++r, ++i) {
                const int cr = cr0 + r;
                // the ring holds rows 2 cr - 3 .. 2 cr + 3 of conv row cr: all seven at a task's first
                // row, then two new rows per conv row (their slots held rows that are long dead)
                if (r == 0) {
                    // a new band reuses ring slots the previous conv row may still be reading: wait
                    // until every producer warp has finished that row's im2col tile
                    if (i > 0 && !mbar_wait(&fullA[(i - 1) & 1], ((i - 1) >> 1) & 1, a.err, s_abort, ERR_WAIT_FULL)) {
                        ok_run = false;
                        break;
                    }
                    for (int y = 2 * cr - 3; y <= 2 * cr + 3; ++y) load_row(n, y);
                } else {
                    load_row(n, 2 * cr + 2);
                    load_row(n, 2 * cr + 3);
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&ringrdy[i & 1]);
                if (!mbar_wait(&ringrdy[i & 1], (i >> 1) & 1, a.err, s_abort, ERR_WAIT_FULL)) { ok_run = false; break; }
                const int b = i & 1;
                if (!mbar_wait(&emptyA[b], ((i >> 1) & 1) ^ 1, a.err, s_abort, ERR_WAIT_EMPTY)) { ok_run = false; break; }
                for (int m = 0; m < MT; ++m) {
                    const int cx = min(m * 128 + pt, CW - 1);     // rows past the conv width: junk
                    const int s2 = 2 * cx;                        // slot start byte in a ring row
                    const int wb = s2 & ~3, sh = (s2 & 3) * 8;
                    uint8_t* tile = sA + (b * MT + m) * ST_KSTEPS * 4096;
                    const int r32 = pt * 32, swz = ((pt >> 2) & 1) << 4;
#pragma unroll
                    for (int kk = 0; kk < ST_KSTEPS; ++kk) {
                        uint32_t wv[8];
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            const int sl = kk * 4 + e;                // slot (ch, ky)
                            if (sl < 21) {
                                const int ch = sl / 7, ky = sl - ch * 7;
                                const int y = 2 * cr + ky - 3;
                                const uint8_t* row = sRing + ((y & (ST_RING - 1)) * 3 + ch) * RB + wb;
                                const uint32_t w0 = *reinterpret_cast<const uint32_t*>(row);
                                const uint32_t w1 = *reinterpret_cast<const uint32_t*>(row + 4);
                                const uint32_t w2 = *reinterpret_cast<const uint32_t*>(row + 8);
                                wv[2 * e] = __funnelshift_r(w0, w1, sh);
                                wv[2 * e + 1] = __funnelshift_r(w1, w2, sh);
                            } else {
                                wv[2 * e] = wv[2 * e + 1] = 0u;
                            }
                        }
                        uint8_t* d = tile + kk * 4096 + r32;
                        *reinterpret_cast<uint4*>(d + swz) = make_uint4(wv[0], wv[1], wv[2], wv[3]);
                        *reinterpret_cast<uint4*>(d + (swz ^ 16)) = make_uint4(wv[4], wv[5], wv[6], wv[7]);
                    }
                }
                fence_async_smem();
                __syncwarp();
                if (lane == 0) mbar_arrive(&fullA[b]);
            }
            if (!ok_run) break;
        }
    } else {
        // ---------------- epilogue: requantise, ring, max-pool ----------------
        const int quad = warp & 3;
        const int et = threadIdx.x - 160;                 // 0..127
        int i = 0;
        for (int t = 0; t < my_tasks; ++t) {
            int n, py0, cr0, nrows;
            task_rows(t, n, py0, cr0, nrows);
            bool ok_run = true;
            for (int r = 0; r < nrows; ++r, ++i) {
                const int cr = cr0 + r;
                const int b = i & 1;
                const int slot = cr % 3;
                // the slot held conv row cr - 3, last read by a pooling done while finishing row i - 1
                if (i > 0 && !mbar_wait(&done[(i - 1) & 1], ((i - 1) >> 1) & 1, a.err, s_abort, ERR_WAIT_EMPTY)) { ok_run = false; break; }
                if (!mbar_wait(&accf[b], (i >> 1) & 1, a.err, s_abort, ERR_WAIT_ACC)) { ok_run = false; break; }
                tc_fence_after();
                for (int m = 0; m < MT; ++m) {
                    const int cx = m * 128 + quad * 32 + lane;
                    uint32_t wd[16];
#pragma unroll
                    for (int cb = 0; cb < 2; ++cb) {
                        uint32_t v[32];
                        const uint32_t taddr = tmem + (static_cast<uint32_t>(quad * 32) << 16) + b * 128 + m * 64 + cb * 32;
                        tmem_ld32(taddr, v);
                        tmem_wait_ld();
                        uint32_t arm[32];
#pragma unroll
                        for (int j = 0; j < 32; ++j) arm[j] = ACC_MAGIC;
                        tmem_st32(taddr, arm);
#pragma unroll
                        for (int j = 0; j < 8; ++j) {
                            uint32_t bq[4];
#pragma unroll
                            for (int e = 0; e < 4; ++e) {
                                const int o = cb * 32 + 4 * j + e;
                                const float f = fast_cvt ? __uint_as_float(v[4 * j + e]) - ACC_MAGIC_F
                                                         : __int2float_rn(static_cast<int32_t>(v[4 * j + e] - ACC_MAGIC));
                                const float tq = fminf(fmaxf(fmaf(f, sKC[o], sKC[64 + o]), 0.0f), 127.0f);
                                bq[e] = __float_as_uint(tq + 12582912.0f);
                            }
                            wd[cb * 8 + j] = __byte_perm(__byte_perm(bq[0], bq[1], 0x0040),
                                                         __byte_perm(bq[2], bq[3], 0x0040), 0x5410);
                        }
                    }
                    if (cx < CW) {
                        // conv ring [3][MT * 128][64 B]; chunk j of pixel p at (j ^ (p & 3)) spreads the banks
                        uint8_t* cp = sC + (static_cast<size_t>(slot) * MT * 128 + cx) * 64;
#pragma unroll
                        for (int j = 0; j < 4; ++j)
                            *reinterpret_cast<uint4*>(cp + ((j ^ (cx & 3)) << 4)) =
                                make_uint4(wd[4 * j], wd[4 * j + 1], wd[4 * j + 2], wd[4 * j + 3]);
                    }
                }
                tmem_wait_st();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(&acce[b]);
                    mbar_arrive(&written[i & 1]);
                }
                // after conv row 2 py + 1: pool pooled row py from conv rows 2py-1 .. 2py+1
                const int py = (cr - 1) >> 1;
                if ((cr & 1) == 1 && py >= py0) {
                    if (!mbar_wait(&written[i & 1], (i >> 1) & 1, a.err, s_abort, ERR_WAIT_ACC)) { ok_run = false; break; }
                    for (int px = et; px < PW; px += 128) {
                        uint32_t mx[16];
#pragma unroll
                        for (int j = 0; j < 16; ++j) mx[j] = 0u;
                        for (int dy = -1; dy <= 1; ++dy) {
                            const int cyy = 2 * py + dy;
                            if (cyy < 0 || cyy >= CH) continue;
                            const uint8_t* rowp = sC + static_cast<size_t>(cyy % 3) * MT * 128 * 64;
                            for (int dx = -1; dx <= 1; ++dx) {
                                const int cxx = 2 * px + dx;
                                if (cxx < 0 || cxx >= CW) continue;
                                const uint8_t* pp = rowp + cxx * 64;
#pragma unroll
                                for (int j = 0; j < 4; ++j) {
                                    const uint4 q = *reinterpret_cast<const uint4*>(pp + ((j ^ (cxx & 3)) << 4));
                                    mx[4 * j] = __vmaxu4(mx[4 * j], q.x);
                                    mx[4 * j + 1] = __vmaxu4(mx[4 * j + 1], q.y);
                                    mx[4 * j + 2] = __vmaxu4(mx[4 * j + 2], q.z);
                                    mx[4 * j + 3] = __vmaxu4(mx[4 * j + 3], q.w);
                                }
                            }
                        }
                        // block 1 input, group-major [2][N][PH * PW][32]
                        const size_t pix = (static_cast<size_t>(n) * PH + py) * PW + px;
                        const size_t gstride = static_cast<size_t>(a.n_alloc > geo.N ? a.n_alloc : geo.N) * PH * PW * 32;
                        int8_t* o = a.out + pix * 32;
                        *reinterpret_cast<uint4*>(o) = make_uint4(mx[0], mx[1], mx[2], mx[3]);
                        *reinterpret_cast<uint4*>(o + 16) = make_uint4(mx[4], mx[5], mx[6], mx[7]);
                        *reinterpret_cast<uint4*>(o + gstride) = make_uint4(mx[8], mx[9], mx[10], mx[11]);
                        *reinterpret_cast<uint4*>(o + gstride + 16) = make_uint4(mx[12], mx[13], mx[14], mx[15]);
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&done[i & 1]);
            }
            if (!ok_run) break;
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_free(tmem, 256);
    }
}

cudaError_t launch_stem(const dn8_stem_args& a, int sms, cudaStream_t st) {
    const StemGeo geo = stem_geo(a.N, a.H, a.W);
    if (geo.smem > 227 * 1024 || a.H % 4 || a.W % 4 || a.W > 512) return cudaErrorInvalidValue;
    const int bands = (geo.PH + ST_BP - 1) / ST_BP;
    const int ntask = a.N * bands;
    const int grid = ntask < sms ? ntask : sms;
    if (grid <= 0) return cudaSuccess;
    cudaError_t e = cudaFuncSetAttribute(stem_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(geo.smem));
    if (e != cudaSuccess) return e;
    stem_kernel<<<grid, ST_THREADS, geo.smem, st>>>(a, geo);
    return cudaGetLastError();
}

}  // namespace dn8
