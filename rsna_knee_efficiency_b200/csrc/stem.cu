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
//              64 + u / 2) in a ring of 14 input rows;
//   warp 0     TMEM owner / MMA issuer: per conv row and M-tile, 7 M128 N64 K32 MMAs (one per
//              kernel row, A = that input row's records) into one of two TMEM accumulators;
//   warps 5-12 (a lane quadrant x a 32-channel half each) requantise their conv pixel's 32
//              channels of each conv row and max-pool as the rows come: each thread owns one conv
//              column (TMEM lane) of every conv row, so the vertical max over conv rows 2py-1 ..
//              2py+1 runs in its registers (16-bit pairs: one vmax2 per two values); the horizontal
//              max over columns 2px-1 .. 2px+1 takes the odd columns' pair max (lane quadrants 2-3:
//              a shuffle, and one edge value across warps) to the even column's thread (quadrants
//              0-1) through a double-buffered exchange in shared memory, which writes the pooled row.
#include <type_traits>

#include "dn8_common.cuh"
#include "dn8_kernels.h"

namespace dn8 {

constexpr int ST_THREADS = 416;          // warp 0 MMA, 1-4 rows + im2col, 5-12 epilogue
constexpr int ST_BP = 16;                 // pooled rows per band
constexpr int ST_RING = 16;               // input row ring
constexpr int ST_KSTEPS = 7;
constexpr int ST_WBYTES = ST_KSTEPS * 64 * 32;   // prepared weights [7][64][32] swizzled
constexpr int ST_REC = 14;                // record ring: input rows y at slot y mod 14
constexpr int MT_MAX = 2;                 // M-tiles of 128 conv pixels per conv row (W <= 512)

struct StemGeo {
    int N, H, W;                           // input
    int CH, CW, PH, PW;                    // conv / pooled output
    int mt;                                // M-tiles per conv row
    int row_bytes;                         // one ring row of one channel: W + 8
    size_t ring_off, rec_off, xo_off, bar_off, smem;
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
    g.xo_off = off; off += static_cast<size_t>(2) * 2 * MT_MAX * 64 * 64 + 2 * 2 * 2 * MT_MAX * 64;   // exchange, edges
    g.bar_off = off; off += 256 + 1024;                                       // kc, barriers
    g.smem = off + 1024;
    return g;
}

// U8: the input is uint8 volume planes (a.x_u8), else fp16 windows; a template parameter, so the row
// prefetch is a plain (predicated) load whose registers nothing reads until the row is put
template <bool U8>
__global__ void __launch_bounds__(ST_THREADS, 1)
stem_kernel(const dn8_stem_args a, const StemGeo geo) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sW = smem;
    uint8_t* sRing = smem + geo.ring_off;
    uint8_t* sRec = smem + geo.rec_off;
    // pooling exchange: odd-column pair maxima [parity][half][M-tile][64 pooled px][16 u16x2 words],
    // then the edge values of lane 31 of quadrants 2 / 3 [parity][half][quadrant - 2][M-tile][16]
    uint32_t* sXo = reinterpret_cast<uint32_t*>(smem + geo.xo_off);
    uint32_t* sXe = sXo + 2 * 2 * MT_MAX * 64 * 16;
    float* sKC = reinterpret_cast<float*>(smem + geo.bar_off);               // [128] k, c
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + geo.bar_off + 512);
    // fullA / emptyA: slot i % 4 for conv row i (the producer runs up to four rows ahead of the MMA)
    uint64_t* fullA = bars;          // [4] the records of conv row i ready (4 producer warps)
    uint64_t* emptyA = bars + 4;     // [4] MMA done with conv row i
    uint64_t* accf = bars + 8;       // [2]
    uint64_t* acce = bars + 10;      // [2] (4 epilogue warps)
    uint64_t* wfull = bars + 12;     // weights landed
    uint64_t* ringrdy = bars + 13;   // [2] input rows of conv row i loaded (4 producer warps)
    uint64_t* eready = bars + 15;    // [2] pooled row k: the edge values published (4 odd-column warps)
    uint64_t* xready = bars + 17;    // [2] pooled row k: the odd columns' pair maxima written (4 warps)
    uint64_t* xfree = bars + 19;     // [2] pooled row k: the exchange read (4 even-column warps)
    uint32_t* s_tmem = reinterpret_cast<uint32_t*>(bars + 21);
    volatile int* s_abort = reinterpret_cast<volatile int*>(s_tmem + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int H = geo.H, W = geo.W, CH = geo.CH, CW = geo.CW, PH = geo.PH, PW = geo.PW, MT = geo.mt;
    const int RB = geo.row_bytes;
    const int bands = (PH + ST_BP - 1) / ST_BP;
    const int ntask = geo.N * bands;
    const int my_tasks = static_cast<int>(blockIdx.x) < ntask ? (ntask - 1 - blockIdx.x) / gridDim.x + 1 : 0;

    if (threadIdx.x == 0) {
        for (int k = 0; k < 2; ++k) {
            mbar_init(&accf[k], 1);
            mbar_init(&acce[k], 8);
            mbar_init(&ringrdy[k], 4);
            mbar_init(&eready[k], 4);
            mbar_init(&xready[k], 4);
            mbar_init(&xfree[k], 4);
        }
        for (int k = 0; k < 4; ++k) {
            mbar_init(&fullA[k], 4);
            mbar_init(&emptyA[k], 1);
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
                    if (!mbar_wait_w(&fullA[i & 3], (i >> 2) & 1, a.err, s_abort, ERR_WAIT_FULL | (67 << 4))) { ok_run = false; break; }
                    tc_fence_after();
                    const int slot0 = ((2 * cr - 3) % ST_REC + ST_REC) % ST_REC;   // records of input row 2 cr - 3
                    for (int m = 0; m < MT; ++m)
#pragma unroll
                        for (int ky = 0; ky < ST_KSTEPS; ++ky) {
                            const int slot = slot0 + ky < ST_REC ? slot0 + ky : slot0 + ky - ST_REC;   // input row's records
                            const uint64_t ad = sdesc(a0 + (slot * MT + m) * 4096, 16, 256, LAYOUT_SW32);
                            const uint64_t bd = sdesc(w0 + ky * 2048, 16, 256, LAYOUT_SW32);
                            umma_u8s8_w(tmem + b * 128 + m * 64, ad, bd, idesc, ky ? 1u : 0u);   // first overwrites
                        }
                    umma_commit_w(&emptyA[i & 3]);
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
        int flip = 0;                                     // the task's image is flipped
        auto fetch = [&](int n, int y, uint2 (&rv)[3]) {
            const bool inside = y >= 0 && y < H && pt < W / 4;
#pragma unroll
            for (int ch = 0; ch < 3; ++ch) {
                rv[ch] = make_uint2(0u, 0u);
                if (inside) {
                    if constexpr (U8) {
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
#pragma unroll
            for (int ch = 0; ch < 3; ++ch) {
                uint32_t v = U8 ? rv[ch].x : (u8_of_f16x2(rv[ch].x) | (u8_of_f16x2(rv[ch].y) << 16));
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
            if constexpr (U8)
#pragma unroll
                for (int ch = 0; ch < 3; ++ch) planes[ch] = a.src[n * 4 + ch];
            flip = a.flags != nullptr ? (a.flags[n] & 1) : 0;      // per image
            bool ok_run = true;
            for (int r = 0; r < nrows; ++r, ++i) {
                const int cr = cr0 + r;
                // the ring holds rows 2 cr - 3 .. 2 cr + 3 of conv row cr: all seven at a task's first
                // row, then two new rows per conv row (their slots held rows that are long dead)
                if (r == 0) {
                    // a new band reuses ring slots the previous conv row may still be reading: wait
                    // until every producer warp has finished that row's im2col tile
                    if (i > 0 && !mbar_wait(&fullA[(i - 1) & 3], ((i - 1) >> 2) & 1, a.err, s_abort, ERR_WAIT_FULL | (68 << 4))) {
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
                // the new records overwrite the slots of input rows 2 cr - 12, 2 cr - 11, last read by
                // conv row i - 4 (at a band's first row, slots of any earlier row: conv row i - 1, whose
                // completion implies every earlier one's): wait until the MMAs of that row are done
                if (!mbar_wait(&emptyA[i & 3], ((i >> 2) & 1) ^ 1, a.err, s_abort, ERR_WAIT_EMPTY | (70 << 4))) { ok_run = false; break; }
                if (r == 0 && i > 0 &&
                    !mbar_wait(&emptyA[(i - 1) & 3], ((i - 1) >> 2) & 1, a.err, s_abort, ERR_WAIT_EMPTY | (71 << 4))) { ok_run = false; break; }
                // records of the new input rows: thread pt builds conv pixels u = 2p and 2p + 1
                // (p = pt % 64) of M-tile pt / 64, as tile rows p and p + 64 (the epilogue maps lane L
                // back to pixel 2L or 2(L - 64) + 1); their 8-byte windows start at ring bytes 2 cx and
                // 2 cx + 2, so three aligned words per channel serve both
                if (pt < MT * 64) {
                    const int m = pt >> 6, r0 = pt & 63;
                    const int wb = 2 * min(m * 128 + 2 * r0, CW - 2);  // pixels past the conv width: junk rows
                    const int swz = ((r0 >> 2) & 1) << 4;
                    auto build = [&](int y) {
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
                    };
                    if (r == 0) {
                        for (int y = 2 * cr - 3; y < 2 * cr + 4; ++y) build(y);
                    } else {
                        // the two new rows: independent loads and stores, issued together
#pragma unroll
                        for (int k2 = 0; k2 < 2; ++k2) build(2 * cr + 2 + k2);
                    }
                }
                fence_async_smem();
                __syncwarp();
                if (lane == 0) mbar_arrive(&fullA[i & 3]);
            }
            if (!ok_run) break;
        }
    } else {
        // ---------------- epilogue: requantise, max-pool ----------------
        // 8 warps: warp w reads TMEM lanes 32 (w % 4) .. + 31 (tile rows: conv pixels) and channel
        // half hc. Tile row r holds conv column 2r (r < 64) or 2(r - 64) + 1 (r >= 64) of each M-tile.
        const int quad = warp & 3, hc = (warp - 5) >> 2;
        const int row = quad * 32 + lane;
        const bool odd = row >= 64;                       // odd conv columns (quadrants 2, 3)
        const int pl = odd ? row - 64 : row;              // pooled pixel within the M-tile
        // the exchange row of pooled pixel pl holds its four 16-byte chunks rotated by pl / 2, so the
        // eight 16-byte accesses of a shared-memory wavefront (pixels pl .. pl + 7, 64 bytes apart)
        // cover all 32 banks
        auto xsw = [&](int j) { return ((((j >> 2) + (pl >> 1)) & 3) << 2); };
        const size_t gstride = static_cast<size_t>(a.n_alloc > geo.N ? a.n_alloc : geo.N) * PH * PW * 32;
        // q = rint(clamp(fmaf(acc, k, c), 0, 127)) of channels 2j, 2j + 1 as the 16-bit pair (q0, q1), with
        // (k, c) of the pair given: int -> float through the magic add (both lanes in one packed add),
        // the packed fma, the clamp, the rounding add of 1.5 * 2^23 (packed) whose low byte is q
        const float2 mneg = make_float2(-ACC_MAGIC_F, -ACC_MAGIC_F), mrnd = make_float2(12582912.0f, 12582912.0f);
        auto requant2 = [&](uint32_t v0, uint32_t v1, float2 k2, float2 c2, auto fast_tag) -> uint32_t {
            float2 f;
            if constexpr (decltype(fast_tag)::value) {
                f = __fadd2_rn(make_float2(__uint_as_float(v0 + ACC_MAGIC), __uint_as_float(v1 + ACC_MAGIC)), mneg);
            } else {
                f = make_float2(__int2float_rn(static_cast<int32_t>(v0)), __int2float_rn(static_cast<int32_t>(v1)));
            }
            float2 t = f2_fma(f, k2, c2);
            t.x = fminf(fmaxf(t.x, 0.0f), 127.0f);
            t.y = fminf(fmaxf(t.y, 0.0f), 127.0f);
            t = __fadd2_rn(t, mrnd);
            return __byte_perm(__float_as_uint(t.x), __float_as_uint(t.y), 0x5410);   // (q0, 0, q1, 0)
        };
        const float4* k4p = reinterpret_cast<const float4*>(sKC + hc * 32);
        const float4* c4p = reinterpret_cast<const float4*>(sKC + 64 + hc * 32);
        // the conversion mode is fixed per launch: one instantiation of the task loop per mode
        auto tasks = [&](auto fast_tag) {
        uint32_t acc[MT_MAX][16];                         // running vertical max of the pooled row
        int i = 0, k = 0;                                 // conv rows, pooled rows of this CTA
        for (int t = 0; t < my_tasks; ++t) {
            int n, py0, cr0, nrows;
            task_rows(t, n, py0, cr0, nrows);
#pragma unroll
            for (int m = 0; m < MT_MAX; ++m)
#pragma unroll
                for (int j = 0; j < 16; ++j) acc[m][j] = 0u;   // the pad row above the image (values >= 0)
            bool ok_run = true;
            for (int r = 0; r < nrows; ++r, ++i) {
                const int cr = cr0 + r;
                const int b = i & 1;
                if (!mbar_wait(&accf[b], (i >> 1) & 1, a.err, s_abort, ERR_WAIT_ACC | (73 << 4))) { ok_run = false; break; }
                tc_fence_after();
                const uint32_t tbase = tmem + (static_cast<uint32_t>(quad * 32) << 16) + b * 128 + hc * 32;
                // conv row 2 py + 1 closes pooled row py (rows 2py-1 .. 2py+1) and opens py + 1
                const bool closes = (cr & 1) == 1;
                const int py = (cr - 1) >> 1;
                uint32_t fin[MT_MAX][16];
#pragma unroll
                for (int j = 0; j < 16; ++j) fin[MT_MAX - 1][j] = 0u;
                // 16 channels (8 pairs) at a time, both M-tiles' columns with the same (k, c)
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    uint32_t v0[16], v1[16];
                    tmem_ld16(tbase + h * 16, v0);
                    if (MT > 1) tmem_ld16(tbase + 64 + h * 16, v1);
                    tmem_wait_ld(v0);
                    reg_bind(v1);
#pragma unroll
                    for (int jq = 0; jq < 4; ++jq) {
                        const float4 k4 = k4p[h * 4 + jq], c4 = c4p[h * 4 + jq];
#pragma unroll
                        for (int e = 0; e < 2; ++e) {
                            const int jj = 2 * jq + e, j = h * 8 + jj;
                            const float2 k2 = e ? make_float2(k4.z, k4.w) : make_float2(k4.x, k4.y);
                            const float2 c2 = e ? make_float2(c4.z, c4.w) : make_float2(c4.x, c4.y);
                            const uint32_t w0 = requant2(v0[2 * jj], v0[2 * jj + 1], k2, c2, fast_tag);
                            fin[0][j] = __vmaxu2(acc[0][j], w0);
                            acc[0][j] = closes ? w0 : fin[0][j];
                            if (MT > 1) {
                                const uint32_t w1 = requant2(v1[2 * jj], v1[2 * jj + 1], k2, c2, fast_tag);
                                fin[1][j] = __vmaxu2(acc[1][j], w1);
                                acc[1][j] = closes ? w1 : fin[1][j];
                            }
                        }
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&acce[b]);          // the accumulator is free
                if (!closes || py < py0) continue;
                // ---- pooled row py: horizontal max over conv columns 2px - 1 .. 2px + 1 ----
                const int par = k & 1, ph = (k >> 1) & 1;
                ++k;
                uint32_t* xo = sXo + (par * 2 + hc) * MT_MAX * 64 * 16;
                uint32_t* xe = sXe + (par * 2 + hc) * 2 * MT_MAX * 16;
                if (odd) {
                    // the exchange of pooled row k - 2 (same parity) has been read
                    if (!mbar_wait(&xfree[par], ph ^ 1, a.err, s_abort, ERR_WAIT_EMPTY | (75 << 4))) { ok_run = false; break; }
                    if (lane == 31) {                          // columns m 128 + 63 (quad 2), m 128 + 127 (quad 3)
#pragma unroll
                        for (int m = 0; m < MT_MAX; ++m)
#pragma unroll
                            for (int j = 0; j < 16; j += 4)
                                *reinterpret_cast<uint4*>(xe + ((quad - 2) * MT_MAX + m) * 16 + j) =
                                    make_uint4(fin[m][j], fin[m][j + 1], fin[m][j + 2], fin[m][j + 3]);
                    }
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&eready[par]);
                    if (!mbar_wait(&eready[par], ph, a.err, s_abort, ERR_WAIT_FULL | (76 << 4))) { ok_run = false; break; }
                    // left neighbour (column 2 pl - 1 of the M-tile): lane - 1, or quad 2's lane 31 (for
                    // quad 3) / quad 3's lane 31 of the previous M-tile (for quad 2; the pad before column 0)
#pragma unroll
                    for (int m = 0; m < MT_MAX; ++m) {
                        const uint32_t* edge = quad == 3 ? xe + (0 * MT_MAX + m) * 16
                                                         : (m > 0 ? xe + (1 * MT_MAX + m - 1) * 16 : nullptr);
#pragma unroll
                        for (int j = 0; j < 16; ++j) {
                            uint32_t left = __shfl_up_sync(0xffffffffu, fin[m][j], 1);
                            if (lane == 0) left = edge != nullptr ? edge[j] : 0u;
                            fin[m][j] = __vmaxu2(fin[m][j], left);
                        }
                        if (m < MT) {
#pragma unroll
                            for (int j = 0; j < 16; j += 4)
                                *reinterpret_cast<uint4*>(xo + (m * 64 + pl) * 16 + xsw(j)) =
                                    make_uint4(fin[m][j], fin[m][j + 1], fin[m][j + 2], fin[m][j + 3]);
                        }
                    }
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&xready[par]);
                } else {
                    if (!mbar_wait(&xready[par], ph, a.err, s_abort, ERR_WAIT_FULL | (77 << 4))) { ok_run = false; break; }
#pragma unroll
                    for (int m = 0; m < MT_MAX; ++m) {
                        if (m >= MT) break;
                        const int px = m * 64 + pl;
                        uint32_t o[16];
#pragma unroll
                        for (int j = 0; j < 16; j += 4) {
                            const uint4 q4 = *reinterpret_cast<const uint4*>(xo + (m * 64 + pl) * 16 + xsw(j));
                            o[j] = q4.x; o[j + 1] = q4.y; o[j + 2] = q4.z; o[j + 3] = q4.w;
                        }
                        uint32_t mx[8];
#pragma unroll
                        for (int j = 0; j < 8; ++j)
                            mx[j] = __byte_perm(__vmaxu2(fin[m][2 * j], o[2 * j]), __vmaxu2(fin[m][2 * j + 1], o[2 * j + 1]),
                                                0x6420);
                        if (px < PW) {
                            // block 1 input, group-major [2][N][PH * PW][32] (this half is group hc), or
                            // groups 0 / 1 of the tile-major block store, whose bytes are q + 128 (q <= 127:
                            // the top bit set)
                            const size_t pix = (static_cast<size_t>(n) * PH + py) * PW + px;
                            const bool tiled = a.tile_groups > 0;
                            const uint32_t ob = tiled ? 0x80808080u : 0u;
                            int8_t* dst = tiled ? a.out + (((pix >> 7) * a.tile_groups + hc) << 12) + (pix & 127) * 32
                                                : a.out + hc * gstride + pix * 32;
                            *reinterpret_cast<uint4*>(dst) = make_uint4(mx[0] | ob, mx[1] | ob, mx[2] | ob, mx[3] | ob);
                            *reinterpret_cast<uint4*>(dst + 16) = make_uint4(mx[4] | ob, mx[5] | ob, mx[6] | ob, mx[7] | ob);
                        }
                    }
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&xfree[par]);
                }
            }
            if (!ok_run) break;
        }
        };
        if (fast_cvt) tasks(std::true_type{});
        else tasks(std::false_type{});
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
    auto kern = a.x_u8 ? stem_kernel<true> : stem_kernel<false>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(geo.smem));
    if (e != cudaSuccess) return e;
    // the first kernel of a pass: its predecessor may be anything (a copy, an event wait)
    return launch_pdl(false, kern, dim3(grid), dim3(ST_THREADS), geo.smem, st, a, geo);
}

}  // namespace dn8
