// stem.cu -- the INT8 stem on sm_100a, fused with the input producer: pixels -> u8 (the uint8
// volume planes directly, or rint(255 sat(x)) of fp16 windows), optional horizontal flip, 7x7/2
// pad-3 conv 3 -> 64 on tcgen05 (kind::i8), q = rint(clamp(fmaf(acc, k, c), 0, 127)), 3x3/2 pad-1
// max-pool on the bytes, into block 1's group-major input [2][N][H/4 * W/4][32] or groups 0-1 of
// its tile-major store.
// Arithmetic of the reference's `stem_i8_body` (src/knee/dense8s_kernels.cu:3641-3771) and
// `stem_q_i8` (src/knee/dense8s.py:625-643).
//
// K layout: the reference's `stem_weights8` (dense8s.py:532-541) has k = (ch * 7 + ky) * 8 + kx',
// kx' = kx + 1 (kx' = 0 has zero weight): slot (ch, ky) of conv pixel cx is the 8 input bytes of
// row 2 cy + ky - 3 starting at column 2 cx - 4. Here the slots are regrouped by kernel row: K step
// ky (32 bytes) = [ch 0 | ch 1 | ch 2 | 8 zero-weight bytes] of input row 2 cy + ky - 3 (7 MMA steps,
// the same products summed in another order, exact in int32). A step depends on the input row
// only, so the 32-byte "record" of every (input row, conv pixel) is built once and serves the
// conv rows that read that input row (up to four).
//
// A CTA walks bands of BP pooled rows of one image; for every conv row of the band (2 BP + 1, the
// first one is the halo shared with the band above):
//   warps 1-4  load the two new input rows (all 3 channels) into a 16-row ring (column c at byte
//              c + 4, four zero bytes either side; the next conv row's loads are issued before this
//              row's records are built), build the records of the new input rows (ceil(CW / 128)
//              M-tiles of 128 pixels x 32 bytes each, 32B-swizzled, pixel u of a tile in row u / 2 or
//              64 + u / 2) in a ring of 10 input rows;
//   warp 0     TMEM owner / MMA issuer: per conv row and M-tile, 7 M128 N64 K32 MMAs (one per
//              kernel row, A = that input row's records) into one of two TMEM accumulators;
//   warps 5-12 (a lane quadrant x a 32-channel half each) requantise into a 3-row ring of conv
//              outputs; after every odd conv row 2 py + 1 they max-pool pooled row py (conv rows
//              2py-1 .. 2py+1) and write it out.
#include "dn8_common.cuh"
#include "dn8_kernels.h"

namespace dn8 {

constexpr int ST_THREADS = 416;          // warp 0 MMA, 1-4 rows + im2col, 5-12 epilogue
constexpr int ST_BP = 16;                 // pooled rows per band
constexpr int ST_RING = 16;               // input row ring
constexpr int ST_KSTEPS = 7;
constexpr int ST_WBYTES = ST_KSTEPS * 64 * 32;   // prepared weights [7][64][32] swizzled
constexpr int ST_REC = 10;                // record ring: input rows y at slot y mod 10

struct StemGeo {
    int N, H, W;                           // input
    int CH, CW, PH, PW;                    // conv / pooled output
    int mt;                                // M-tiles per conv row
    int row_bytes;                         // one ring row of one channel: W + 8
    size_t ring_off, rec_off, conv_off, bar_off, smem;
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
    g.rec_off = off; off += static_cast<size_t>(ST_REC) * g.mt * 4096;        // record ring
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
    uint8_t* sRec = smem + geo.rec_off;
    uint8_t* sC = smem + geo.conv_off;
    float* sKC = reinterpret_cast<float*>(smem + geo.bar_off);               // [128] k, c
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + geo.bar_off + 512);
    uint64_t* fullA = bars;          // [2] the records of conv row i ready (4 producer warps)
    uint64_t* emptyA = bars + 2;     // [2] MMA done with conv row i (by row parity)
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
            mbar_init(&acce[k], 8);
            mbar_init(&ringrdy[k], 4);
            mbar_init(&written[k], 8);
            mbar_init(&done[k], 8);
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
    tc_fence_before();
    const int fast_cvt = __syncthreads_and(ok);
    tc_fence_after();
    griddep_launch_dependents();
    griddep_wait();                                    // pixels, and the readers of block 1's input

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
        // ---------------- MMA issuer (the whole warp; one elected lane issues) ----------------
        if (my_tasks > 0) {
            if (lane == 0) {
                mbar_expect_tx(&wfull[0], ST_WBYTES);
                bulk_g2s(sW, a.w, ST_WBYTES, &wfull[0]);
            }
            __syncwarp();
            bool ok_run = mbar_wait_w(&wfull[0], 0, a.err, s_abort, ERR_WAIT_FULL | (65 << 4));
            const uint32_t idesc = idesc_u8s8(128, 64);
            const uint32_t a0 = smem_u32(sRec), w0 = smem_u32(sW);
            int i = 0;
            for (int t = 0; t < my_tasks && ok_run; ++t) {
                int n, py0, cr0, nrows;
                task_rows(t, n, py0, cr0, nrows);
                for (int r = 0; r < nrows; ++r, ++i) {
                    const int b = i & 1, cr = cr0 + r;
                    if (!mbar_wait_w(&acce[b], ((i >> 1) & 1) ^ 1, a.err, s_abort, ERR_WAIT_ACC | (66 << 4))) { ok_run = false; break; }
                    if (!mbar_wait_w(&fullA[b], (i >> 1) & 1, a.err, s_abort, ERR_WAIT_FULL | (67 << 4))) { ok_run = false; break; }
                    tc_fence_after();
                    for (int m = 0; m < MT; ++m)
#pragma unroll
                        for (int ky = 0; ky < ST_KSTEPS; ++ky) {
                            const int slot = ((2 * cr + ky - 3) % ST_REC + ST_REC) % ST_REC;   // input row's records
                            const uint64_t ad = sdesc(a0 + (slot * MT + m) * 4096, 16, 256, LAYOUT_SW32);
                            const uint64_t bd = sdesc(w0 + ky * 2048, 16, 256, LAYOUT_SW32);
                            umma_u8s8_w(tmem + b * 128 + m * 64, ad, bd, idesc, ky ? 1u : 0u);   // first overwrites
                        }
                    umma_commit_w(&emptyA[b]);
                    umma_commit_w(&accf[b]);
                }
            }
        }
        __syncwarp();
    } else if (warp <= 4) {
        // ---------------- input rows + im2col ----------------
        const int pt = threadIdx.x - 32;                  // 0..127
        // Input row y (all 3 channels) of image n: fetched into registers (one word of 4 pixels,
        // or four fp16 pixels, per channel and thread; the loads of a row are independent), then
        // put into ring slot y % ST_RING (column c at byte c + 4, flipped if asked).
        int planes[3] = {0, 0, 0};                        // uint8 planes of the task's image
        auto fetch = [&](int n, int y, uint2 (&rv)[3]) {
            const bool inside = y >= 0 && y < H && pt < W / 4;
#pragma unroll
            for (int ch = 0; ch < 3; ++ch) {
                rv[ch] = make_uint2(0u, 0u);
                if (inside) {
                    if (a.x_u8) {
                        rv[ch].x = __ldg(reinterpret_cast<const uint32_t*>(static_cast<const uint8_t*>(a.x) +
                                                                             (static_cast<size_t>(planes[ch]) * H + y) * W) + pt);
                    } else {
                        rv[ch] = __ldg(reinterpret_cast<const uint2*>(static_cast<const uint16_t*>(a.x) +
                                                                      ((static_cast<size_t>(n) * 3 + ch) * H + y) * W) + pt);
                    }
                }
            }
        };
        auto put = [&](int n, int y, const uint2 (&rv)[3]) {
            if (pt >= W / 4) return;
            uint8_t* dst = sRing + (y & (ST_RING - 1)) * 3 * RB + 4;
            const int flip = a.flags != nullptr ? (a.flags[n] & 1) : 0;
#pragma unroll
            for (int ch = 0; ch < 3; ++ch) {
                uint32_t v = a.x_u8 ? rv[ch].x : (u8_of_f16x2(rv[ch].x) | (u8_of_f16x2(rv[ch].y) << 16));
                int col = 4 * pt;
                if (flip) {
                    v = __byte_perm(v, 0, 0x0123);
                    col = W - 4 - col;
                }
                *reinterpret_cast<uint32_t*>(dst + ch * RB + col) = v;
            }
        };
        int i = 0;
        uint2 pre0[3], pre1[3];                           // the next conv row's two input rows
        for (int t = 0; t < my_tasks; ++t) {
            int n, py0, cr0, nrows;
            task_rows(t, n, py0, cr0, nrows);
            if (a.x_u8)
#pragma unroll
                for (int ch = 0; ch < 3; ++ch) planes[ch] = a.src[n * 4 + ch];
            bool ok_run = true;
            for (int r = 0; r < nrows; ++r, ++i) {
                const int cr = cr0 + r;
                // the ring holds rows 2 cr - 3 .. 2 cr + 3 of conv row cr: all seven at a task's first
                // row, then two new rows per conv row (their slots held rows that are long dead)
                if (r == 0) {
                    // a new band reuses ring slots the previous conv row may still be reading: wait
                    // until every producer warp has finished that row's im2col tile
                    if (i > 0 && !mbar_wait(&fullA[(i - 1) & 1], ((i - 1) >> 1) & 1, a.err, s_abort, ERR_WAIT_FULL | (68 << 4))) {
                        ok_run = false;
                        break;
                    }
                    for (int k = 0; k < 7; k += 2) {              // two rows' loads in flight at a time
                        fetch(n, 2 * cr - 3 + k, pre0);
                        if (k + 1 < 7) fetch(n, 2 * cr - 2 + k, pre1);
                        put(n, 2 * cr - 3 + k, pre0);
                        if (k + 1 < 7) put(n, 2 * cr - 2 + k, pre1);
                    }
                } else {
                    put(n, 2 * cr + 2, pre0);
                    put(n, 2 * cr + 3, pre1);
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&ringrdy[i & 1]);
                if (!mbar_wait(&ringrdy[i & 1], (i >> 1) & 1, a.err, s_abort, ERR_WAIT_FULL | (69 << 4))) { ok_run = false; break; }
                // the next conv row's input rows load while this row's im2col tile is built
                if (r + 1 < nrows) {
                    fetch(n, 2 * cr + 4, pre0);
                    fetch(n, 2 * cr + 5, pre1);
                }
                const int b = i & 1;
                // the new records overwrite the slots last read by conv row i - 2 (and, at a band's
                // first row, by conv row i - 1 too): wait until the MMAs of those rows are done
                if (!mbar_wait(&emptyA[b], ((i >> 1) & 1) ^ 1, a.err, s_abort, ERR_WAIT_EMPTY | (70 << 4))) { ok_run = false; break; }
                if (r == 0 && i > 0 &&
                    !mbar_wait(&emptyA[(i - 1) & 1], ((i - 1) >> 1) & 1, a.err, s_abort, ERR_WAIT_EMPTY | (71 << 4))) { ok_run = false; break; }
                // records of the new input rows: thread pt builds conv pixels u = 2p and 2p + 1
                // (p = pt % 64) of M-tile pt / 64, as tile rows p and p + 64 (the epilogue maps lane L
                // back to pixel 2L or 2(L - 64) + 1); their 8-byte windows start at ring bytes 2 cx and
                // 2 cx + 2, so three aligned words per channel serve both
                if (pt < MT * 64) {
                    const int m = pt >> 6, r0 = pt & 63;
                    const int wb = 2 * min(m * 128 + 2 * r0, CW - 2);  // pixels past the conv width: junk rows
                    const int swz = ((r0 >> 2) & 1) << 4;
                    const int y_first = r == 0 ? 2 * cr - 3 : 2 * cr + 2;
                    const int y_end = 2 * cr + 4;
                    for (int y = y_first; y < y_end; ++y) {
                        uint32_t w0v[6], w1v[6];
#pragma unroll
                        for (int ch = 0; ch < 3; ++ch) {
                            const uint8_t* row = sRing + ((y & (ST_RING - 1)) * 3 + ch) * RB + wb;
                            const uint32_t u0 = *reinterpret_cast<const uint32_t*>(row);
                            const uint32_t u1 = *reinterpret_cast<const uint32_t*>(row + 4);
                            const uint32_t u2 = *reinterpret_cast<const uint32_t*>(row + 8);
                            w0v[2 * ch] = u0;
                            w0v[2 * ch + 1] = u1;
                            w1v[2 * ch] = __funnelshift_r(u0, u1, 16);
                            w1v[2 * ch + 1] = __funnelshift_r(u1, u2, 16);
                        }
                        const int slot = (y % ST_REC + ST_REC) % ST_REC;
                        uint8_t* d0 = sRec + (slot * MT + m) * 4096 + r0 * 32;
                        *reinterpret_cast<uint4*>(d0 + swz) = make_uint4(w0v[0], w0v[1], w0v[2], w0v[3]);
                        *reinterpret_cast<uint4*>(d0 + (swz ^ 16)) = make_uint4(w0v[4], w0v[5], 0u, 0u);
                        uint8_t* d1 = d0 + 64 * 32;
                        *reinterpret_cast<uint4*>(d1 + swz) = make_uint4(w1v[0], w1v[1], w1v[2], w1v[3]);
                        *reinterpret_cast<uint4*>(d1 + (swz ^ 16)) = make_uint4(w1v[4], w1v[5], 0u, 0u);
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
        // 8 warps: warp w reads TMEM lanes 32 (w % 4) .. + 31 (conv pixels) and channel half hc;
        // the pooling splits the pooled pixels x channel halves (= the two output groups) likewise.
        const int quad = warp & 3, hc = (warp - 5) >> 2;
        const int et = threadIdx.x - 160;                 // 0..255
        const int pxh = et & 1, px0 = et >> 1;            // pooling: channel half, first pooled pixel
        const size_t gstride = static_cast<size_t>(a.n_alloc > geo.N ? a.n_alloc : geo.N) * PH * PW * 32;
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
                if (i > 0 && !mbar_wait(&done[(i - 1) & 1], ((i - 1) >> 1) & 1, a.err, s_abort, ERR_WAIT_EMPTY | (72 << 4))) { ok_run = false; break; }
                if (!mbar_wait(&accf[b], (i >> 1) & 1, a.err, s_abort, ERR_WAIT_ACC | (73 << 4))) { ok_run = false; break; }
                tc_fence_after();
                // both M-tiles of the conv row (MT <= 2): their TMEM loads issued together, each (k, c)
                // quad read once for both
                const int row = quad * 32 + lane;              // tile row -> conv pixel (see im2col)
                const int cxr = row < 64 ? 2 * row : 2 * (row - 64) + 1;
                const uint32_t tbase = tmem + (static_cast<uint32_t>(quad * 32) << 16) + b * 128 + hc * 32;
                uint32_t v0[32], v1[32];
                tmem_ld32(tbase, v0);
                if (MT > 1) tmem_ld32(tbase + 64, v1);
                tmem_wait_ld(v0);
                reg_bind(v1);
                // q = rint(clamp(fmaf(acc, k, c), 0, 127)) of 4 channels as the bytes of one word
                auto requant4 = [&](const uint32_t (&v)[32], int j, const float4& k4, const float4& c4) -> uint32_t {
                    float f[4];
#pragma unroll
                    for (int e = 0; e < 4; ++e)
                        f[e] = fast_cvt ? __uint_as_float(v[4 * j + e] + ACC_MAGIC) - ACC_MAGIC_F
                                        : __int2float_rn(static_cast<int32_t>(v[4 * j + e]));
                    float tq[4];
                    f2_unpack(f2_fma(f2_pack(f[0], f[1]), f2_pack(k4.x, k4.y), f2_pack(c4.x, c4.y)), tq[0], tq[1]);
                    f2_unpack(f2_fma(f2_pack(f[2], f[3]), f2_pack(k4.z, k4.w), f2_pack(c4.z, c4.w)), tq[2], tq[3]);
                    uint32_t bq[4];
#pragma unroll
                    for (int e = 0; e < 4; ++e)
                        bq[e] = __float_as_uint(fminf(fmaxf(tq[e], 0.0f), 127.0f) + 12582912.0f);
                    return __byte_perm(__byte_perm(bq[0], bq[1], 0x0040), __byte_perm(bq[2], bq[3], 0x0040), 0x5410);
                };
                uint32_t wd0[8], wd1[8];
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    // k, c of the 4 channels (broadcast reads); fmaf pairwise in f32x2
                    const float4 k4 = *reinterpret_cast<const float4*>(sKC + hc * 32 + 4 * j);
                    const float4 c4 = *reinterpret_cast<const float4*>(sKC + 64 + hc * 32 + 4 * j);
                    wd0[j] = requant4(v0, j, k4, c4);
                    wd1[j] = MT > 1 ? requant4(v1, j, k4, c4) : 0u;
                }
                // conv ring [3][MT][128 tile rows][64 B], by tile row; chunk j of row r at (j ^ (r & 3))
                // spreads the banks
                auto put_row = [&](int m, const uint32_t (&wd)[8]) {
                    if (m * 128 + cxr >= CW) return;
                    uint8_t* cp = sC + (static_cast<size_t>(slot) * MT * 128 + m * 128 + row) * 64;
#pragma unroll
                    for (int j = 0; j < 2; ++j)
                        *reinterpret_cast<uint4*>(cp + (((2 * hc + j) ^ (row & 3)) << 4)) =
                            make_uint4(wd[4 * j], wd[4 * j + 1], wd[4 * j + 2], wd[4 * j + 3]);
                };
                put_row(0, wd0);
                if (MT > 1) put_row(1, wd1);
                tc_fence_before();
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(&acce[b]);
                    mbar_arrive(&written[i & 1]);
                }
                // after conv row 2 py + 1: pool pooled row py from conv rows 2py-1 .. 2py+1
                const int py = (cr - 1) >> 1;
                if ((cr & 1) == 1 && py >= py0) {
                    if (!mbar_wait(&written[i & 1], (i >> 1) & 1, a.err, s_abort, ERR_WAIT_ACC | (74 << 4))) { ok_run = false; break; }
                    for (int px = px0; px < PW; px += 128) {
                        // per-byte max of the 9 taps as u16x2 max of the even and the odd bytes of
                        // every word (one native instruction each; a 4-byte SIMD max is not native)
                        uint32_t mxe[8], mxo[8];
#pragma unroll
                        for (int j = 0; j < 8; ++j) mxe[j] = mxo[j] = 0u;
#pragma unroll
                        for (int dy = -1; dy <= 1; ++dy) {
                            const int cyy = 2 * py + dy;
                            if (cyy < 0 || cyy >= CH) continue;
                            const uint8_t* rowp = sC + static_cast<size_t>(cyy % 3) * MT * 128 * 64;
#pragma unroll
                            for (int dx = -1; dx <= 1; ++dx) {
                                const int cxx = 2 * px + dx;
                                if (cxx < 0 || cxx >= CW) continue;
                                const int u = cxx & 127;
                                const int trow = (u & 1) ? 64 + (u >> 1) : (u >> 1);
                                const uint8_t* pp = rowp + ((cxx >> 7) * 128 + trow) * 64;
#pragma unroll
                                for (int j = 0; j < 2; ++j) {
                                    const uint4 q = *reinterpret_cast<const uint4*>(pp + (((2 * pxh + j) ^ (trow & 3)) << 4));
                                    const uint32_t qw[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
                                    for (int k = 0; k < 4; ++k) {
                                        mxe[4 * j + k] = __vmaxu2(mxe[4 * j + k], __byte_perm(qw[k], 0u, 0x4240));
                                        mxo[4 * j + k] = __vmaxu2(mxo[4 * j + k], __byte_perm(qw[k], 0u, 0x4341));
                                    }
                                }
                            }
                        }
                        // block 1 input, group-major [2][N][PH * PW][32] (this half is group pxh), or
                        // groups 0 / 1 of the tile-major block store
                        const size_t pix = (static_cast<size_t>(n) * PH + py) * PW + px;
                        int8_t* o = a.tile_groups > 0
                                        ? a.out + (((pix >> 7) * a.tile_groups + pxh) << 12) + (pix & 127) * 32
                                        : a.out + pxh * gstride + pix * 32;
                        uint32_t mx[8];
#pragma unroll
                        for (int j = 0; j < 8; ++j) mx[j] = __byte_perm(mxe[j], mxo[j], 0x6240);
                        *reinterpret_cast<uint4*>(o) = make_uint4(mx[0], mx[1], mx[2], mx[3]);
                        *reinterpret_cast<uint4*>(o + 16) = make_uint4(mx[4], mx[5], mx[6], mx[7]);
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
    // the first kernel of a pass: its predecessor may be anything (a copy, an event wait)
    return launch_pdl(false, stem_kernel, dim3(grid), dim3(ST_THREADS), geo.smem, st, a, geo);
}

}  // namespace dn8
