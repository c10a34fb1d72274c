// gemm.cu -- the "prologue GEMM" kernels of the encoder on sm_100a: conv1 of every dense layer and
// the transitions. Both read a block store of 32-channel int8 groups -- group-major planes
// [G][N][HW][32] (block input groups first, then the layer segments: the reference's layout, at the
// kernel ABI) or tile-major [ceil(N HW / 128)][tg][128][32] (all groups of 128 consecutive pixels
// contiguous: the engine's layout) -- apply the consumer's BatchNorm + ReLU + u8 quantisation (the
// prologue), multiply on tcgen05 (kind::i8, u8 x s8 -> s32 in TMEM) and requantise in the epilogue.
//
//   conv1      : M = N*HW pixels, N = 128, K = c_in; out = rint(255 sat(g acc + d)) as the u8
//                bottleneck planes [8][M][16] (reference conv1w_body, dense8s_kernels.cu:479-627).
//   transition : M = N*HW/4 pooled pixels, N = c_out (chunks of 128 or 256), K = c_tot. For every
//                K group the four pixels of each 2x2 square are four A sub-tiles multiplied by the
//                same weights into ONE accumulator: s = the sum of the four 1x1 outputs, exact in
//                int32 (the integer form gemm_q MODE 1, :375-389); q = rint(clamp(k s, +-127)) into
//                the next block's group-major input [c_out/32][N][HW/4][32] or tile-major store.
//
// Pipeline stage = 4 "units" of 128 rows x 32 bytes (16 KB of A, 4 MMAs M128 x NC x K32, one
// commit): conv1 takes 4 consecutive K groups per stage, the transition the 4 pixels of each
// square of one K group. Each MMA issue costs ~80 cycles even from a converged warp, so issuing 4
// MMAs per wait / commit is what keeps the tensor core fed. The store bytes of a stage
// arrive by bulk async copies into a shared-memory ring (explicit bytes in flight, no L1 staging).
// Persistent, one CTA per SM, 19 warps:
//   warp 0       TMEM owner and MMA issuer (the whole warp; one elected lane issues).
//   warp 1       store producer: bulk copies into the raw ring (tile-major: one copy per stage;
//                group-major: one lane per K group of a stage; the transition: one per 4 KB tile).
//   warp 2       weight producer (lane 0): UMMA-ready weight tiles, resident when they fit.
//   warps 3-10   prologue: raw ring -> BN/ReLU/u8 -> the A operand (conv1: TMEM, two warps per
//                lane quadrant taking alternate stages; transition: one warp per unit, 32B-swizzled
//                shared memory).
//   warps 11-18  epilogue: warp w reads TMEM lanes 32*(w%4).. and half of the NC columns.
// conv1 layers whose weights do not fit one CTA run on CTA pairs (clusters of two, PAIR): 256-row
// tiles, CTA r holding rows 128 r .. and the weights of output channels 64 r ..; the even CTA's
// warp 0 issues M = 256 MMAs over both CTAs (tcgen05 cta_group::2), the odd CTA's prologue and
// epilogue warps arrive on the even CTA's fullA / acce, and commits arrive in both CTAs.
#include <atomic>
#include <type_traits>

#include "dn8_common.cuh"
#include "dn8_kernels.h"

namespace dn8 {

constexpr int GM_WARPS = 19;
constexpr int GM_THREADS = 32 * GM_WARPS;
constexpr int SMEM_BUDGET = 225 * 1024;

// KSTEP K groups of KSUB sub-tiles per stage (KSTEP * KSUB = 4 units); SR raw slots (the transition's;
// conv1 sizes its ring at launch), SA operand slots
template <bool TRANS> struct GemmCfg;
// conv1 keeps its A operands in TMEM (columns 256..511 behind the two 128-column accumulators:
// SA = 8 stages of 4 units x 8 columns); the transition (NC up to 256 accumulator columns) keeps
// them in shared memory.
template <> struct GemmCfg<false> {                // conv1
    static constexpr int KSUB = 1, KSTEP = 4, SA = 8;
    static constexpr bool TMEM_A = true;
};
template <> struct GemmCfg<true> {                 // transition
    static constexpr int KSUB = 4, KSTEP = 1, SR = 4, SA = 4;
    static constexpr bool TMEM_A = false;
};
constexpr uint32_t TMEM_A_COL = 256;               // conv1: first TMEM column of the A stages
constexpr int UNITS = 4;

struct GemmArgs {
    const int8_t* in0;        // block input groups [G0][N][HW][32]
    const int8_t* seg;        // layer segments [L][N][HW][32]
    const uint8_t* wu;        // UMMA-ready weights [nchunks][G][chunk rows x 32 B, 32B-swizzled]
    const void* ab;           // prologue table (fp16 pairs or fp32 pairs)
    const float* gd;          // epilogue table [cout][2]
    void* out;
    int* err;
    int G0, G, N, HW, W;      // W: image width (transition)
    int rows;                 // GEMM rows: N*HW (conv1) or N*HW/4 (transition)
    int cout, nc, nchunks;    // output channels, channels per chunk (the last one may be 128), chunks
    int b_resident;           // 1: all G weight tiles stay in shared memory
    int sb;                   // weight ring stages when streamed
    int raw_bytes;            // raw ring slot size (a whole stage)
    int sr;                   // raw ring slots
    int tg;                   // 0 = group-major planes; > 0 = tile-major input store with tg groups per tile
    int tg_out;               // transition: 0 = group-major output; > 0 = the next block's tile-major store
    long long wait_limit;     // SM cycles a wait may take before the launch gives up (WAIT_LIMIT)
    int fault;                // test hook (dn8_test_inject_wait_fault): 1 = the store producer of the first
                              // CTA (pair) never posts raw stage 0 of its first tile, so a wait runs out
};

// Byte range [first, end) of the flattened input pixels (n * HW + y * W + x) a transition tile of
// pooled pixels [m0, m0 + cnt) reads: whole input rows from 2 * oy(first) to 2 * oy(last) + 1.
DN8_DEV void trans_span(int m0, int cnt, int HW, int W, int* first, int* end) {
    const int HW4 = HW >> 2, W2 = W >> 1;
    const int n0 = m0 / HW4, oy0 = (m0 - n0 * HW4) / W2;
    const int m1 = m0 + cnt - 1;
    const int n1 = m1 / HW4, oy1 = (m1 - n1 * HW4) / W2;
    *first = n0 * HW + 2 * oy0 * W;
    *end = n1 * HW + (2 * oy1 + 2) * W;
}

// conv1's raw ring takes what shared memory is left after the weights (at least CONV1_SR_MIN and at
// most CONV1_SR_MAX stages of 16 KB): with many K groups per tile a stage is held ~1,500 cycles by
// the prologue, and four slots (64 KB in flight per SM) cap the store stream near 3 TB/s.
constexpr int CONV1_SR_MIN = 4, CONV1_SR_MAX = 12;

static size_t gemm_layout(bool trans, bool pair, int G, int nc, int nchunks, int raw_bytes, int* sb, int* resident,
                          int* sr_out) {
    const int sr = trans ? GemmCfg<true>::SR : CONV1_SR_MIN, sa = trans ? GemmCfg<true>::SA : GemmCfg<false>::SA;
    const int kstep = trans ? GemmCfg<true>::KSTEP : GemmCfg<false>::KSTEP;
    const size_t a_smem = trans ? static_cast<size_t>(sa) * UNITS * 4096 : 0;     // conv1: A in TMEM
    const size_t fixed = static_cast<size_t>(sr) * raw_bytes + a_smem;
    const size_t misc = 1024 + static_cast<size_t>(G) * 256 + static_cast<size_t>(trans ? 640 : 128) * 8 + 8 * 96 + 64;
    const size_t btile = static_cast<size_t>(pair ? nc / 2 : nc) * 32;   // a CTA of a pair holds half
    size_t used;
    if (nchunks == 1 && fixed + misc + btile * G <= SMEM_BUDGET) {
        *resident = 1;
        *sb = G;
        used = fixed + misc + btile * G;
    } else {
        *resident = 0;
        // streamed: a ring of `s` stages of kstep weight tiles
        int s = static_cast<int>((SMEM_BUDGET - fixed - misc) / (btile * kstep));
        s = s > 4 ? 4 : s;
        *sb = s;
        used = fixed + misc + btile * kstep * s;
    }
    *sr_out = sr;
    if (!trans && used <= SMEM_BUDGET) {
        int extra = static_cast<int>((SMEM_BUDGET - used) / raw_bytes);
        extra = extra > CONV1_SR_MAX - sr ? CONV1_SR_MAX - sr : extra;
        // An even ring: slot s then only ever carries stages of one parity, i.e. of one of the two
        // prologue warps of a lane quadrant, and that warp waits on the slot's phases one after the
        // other. With an odd ring the other warp could start waiting on stage i while stage i - SR of
        // the same slot (an earlier copy, not yet landed) is still the slot's open phase; a parity
        // wait two phases ahead passes at once, and the warp would read the slot before its bytes.
        extra &= ~1;
        *sr_out = sr + extra;
        used += static_cast<size_t>(extra) * raw_bytes;
    }
    return used;
}

template <bool F16, bool TRANS, bool PAIR, bool OB>
__global__ void __launch_bounds__(GM_THREADS, 1) gemm_kernel(const GemmArgs a) {
    using Cfg = GemmCfg<TRANS>;
    // OB: the input store is tile-major and holds q + 128 per byte (offset binary), the prologue's
    // own input form; group-major planes hold signed q, flipped to it by one xor per 4 bytes
    constexpr uint32_t XM = OB ? 0u : 0x80808080u;
    constexpr int KSTEP = Cfg::KSTEP, SA = Cfg::SA;
    const int SR = TRANS ? GemmCfg<true>::SR : a.sr;            // transition: a fixed 4-stage ring
    constexpr int ASTAGE = UNITS * 4096;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    // PAIR (conv1 whose weights do not fit one CTA): CTA pairs, a tile is 256 rows, rows 128 r .. of
    // it in CTA r, whose shared memory holds the weights of output channels 64 r .. + 63 (a 2 KB half
    // of each K group's tile)
    static_assert(!(PAIR && TRANS), "the transition runs on single CTAs");
    const int NC = a.nc, G = a.G, G0 = a.G0, HW = a.HW, rows = a.rows;
    const int btile = (PAIR ? NC / 2 : NC) * 32, RB = a.raw_bytes;   // this CTA's weight tile bytes
    constexpr bool TMEM_A = Cfg::TMEM_A;
    constexpr int MT = PAIR ? 256 : 128;                         // rows per tile
    const uint32_t rank = PAIR ? cluster_rank() : 0u;
    const int unit = PAIR ? static_cast<int>(blockIdx.x >> 1) : static_cast<int>(blockIdx.x);   // pair / CTA
    const int nunits = PAIR ? static_cast<int>(gridDim.x >> 1) : static_cast<int>(gridDim.x);
    uint8_t* sR = smem;                                          // [SR][RB] raw store bytes
    uint8_t* sA = sR + SR * RB;                                  // [SA][KSUB][128][32] swizzled (transition)
    uint8_t* sB = sA + (TMEM_A ? 0 : SA * ASTAGE);               // weights
    const int bstage = KSTEP * btile;                            // weight bytes of a streamed stage
    uint8_t* sTab = sB + (a.b_resident ? static_cast<size_t>(G) * btile : static_cast<size_t>(a.sb) * bstage);
    float2* sGd = reinterpret_cast<float2*>(sTab + G * 256);
    uint64_t* fullR = reinterpret_cast<uint64_t*>(sGd + (TRANS ? 640 : 128));
    uint64_t* freeR = fullR + SR;
    uint64_t* fullA = freeR + SR;
    uint64_t* emptyA = fullA + SA;
    uint64_t* fullB = emptyA + SA;                               // [8]
    uint64_t* emptyB = fullB + 8;
    uint64_t* accf = emptyB + 8;
    uint64_t* acce = accf + 2;
    uint32_t* s_tmem = reinterpret_cast<uint32_t*>(acce + 2);
    volatile int* s_abort = reinterpret_cast<volatile int*>(s_tmem + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const long long lim = a.wait_limit;
    const int ntm = (rows + MT - 1) / MT;
    const int ntiles = ntm * a.nchunks;
    const int my_tiles = unit < ntiles ? (ntiles - 1 - unit) / nunits + 1 : 0;
    const int NS = (G + KSTEP - 1) / KSTEP;                     // stages per tile
    const int T = my_tiles * NS;
    const uint32_t tcols = (NC > 128 || TMEM_A) ? 512u : 256u;
    const size_t gstride = static_cast<size_t>(a.N) * HW * 32;   // one store group

    if (threadIdx.x == 0) {
        for (int s = 0; s < SR; ++s) {
            mbar_init(&fullR[s], 1);
            mbar_init(&freeR[s], UNITS);
        }
        for (int s = 0; s < SA; ++s) {
            mbar_init(&fullA[s], PAIR ? 2 * UNITS : UNITS);        // pair: both CTAs' quadrant warps
            mbar_init(&emptyA[s], 1);
        }
        for (int s = 0; s < 8; ++s) {
            mbar_init(&fullB[s], 1);
            mbar_init(&emptyB[s], 1);
        }
        for (int k = 0; k < 2; ++k) {
            mbar_init(&accf[k], 1);
            mbar_init(&acce[k], PAIR ? 16 : 8);                     // pair: both CTAs' epilogue warps
        }
        *s_abort = 0;
        mbar_fence_init();
    }
    if (F16) {
        for (int i = threadIdx.x; i < G * 16; i += GM_THREADS)
            reinterpret_cast<uint2*>(sTab)[i] = reinterpret_cast<const uint2*>(a.ab)[i];
    } else {
        for (int i = threadIdx.x; i < G * 32; i += GM_THREADS)
            reinterpret_cast<float2*>(sTab)[i] = reinterpret_cast<const float2*>(a.ab)[i];
    }
    // The epilogue converts int32 -> float with the 1.5 * 2^23 magic add, exact for |acc| < 2^22.
    // Larger accumulators convert to values of the same sign and magnitude >= 2^22; that is
    // harmless when every channel already saturates at +-2^22, which is checked here per CTA.
    int ok = 1;
    for (int i = threadIdx.x; i < a.cout; i += GM_THREADS) {
        const float2 p = reinterpret_cast<const float2*>(a.gd)[i];
        if (TRANS) {
            sGd[i] = p;
        } else {                                      // conv1: (g0, g1, d0, d1) per channel pair
            float* q = reinterpret_cast<float*>(sGd) + 4 * (i >> 1) + (i & 1);
            q[0] = p.x;
            q[2] = p.y;
        }
        if (TRANS) ok &= (p.x * 4194304.0f >= 127.0f) ? 1 : 0;
        else ok &= (fmaf(p.x, 4194304.0f, p.y) >= 1.0f && fmaf(p.x, -4194304.0f, p.y) <= 0.0f) ? 1 : 0;
    }
    if (warp == 0) {
        if constexpr (PAIR) tmem_alloc_pair(s_tmem, tcols);
        else tmem_alloc(s_tmem, tcols);
    }
    tc_fence_before();
    if constexpr (PAIR) cluster_sync();               // also: both CTAs' barriers initialised
    else __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *s_tmem;
    tc_fence_before();
    const int fast_cvt = __syncthreads_and(ok);
    tc_fence_after();
    if (warp == 2 && lane == 0 && T > 0 && a.b_resident) {
        // resident weights (constant: they may land while the previous kernel still runs)
        mbar_expect_tx(&fullB[0], static_cast<uint32_t>(G * btile));
        if constexpr (PAIR) {
            for (int g = 0; g < G; ++g)                       // this CTA's half of each K group's tile
                bulk_g2s(sB + g * btile, a.wu + static_cast<size_t>(g) * 2 * btile + rank * btile,
                         static_cast<uint32_t>(btile), &fullB[0]);
        } else {
            bulk_g2s(sB, a.wu, static_cast<uint32_t>(G * btile), &fullB[0]);
        }
    }
    griddep_launch_dependents();
    griddep_wait();                                    // the previous layer's store / bottleneck

    if (warp == 0) {
        if (!PAIR || rank == 0) {
            // ---------------- MMA issuer (the whole warp; one elected lane issues) ----------------
            // pair: the even CTA issues for both; its fullA / acce count both CTAs' warps, and every
            // commit arrives in both CTAs
            const uint32_t a0 = smem_u32(sA), b0 = smem_u32(sB);
            bool ok_run = true;
            if (a.b_resident && T > 0) {
                ok_run = mbar_wait_w(&fullB[0], 0, a.err, s_abort, ERR_WAIT_FULL | (1 << 4), lim);
                if (PAIR && ok_run) ok_run = mbar_wait_w(&fullB[1], 0, a.err, s_abort, ERR_WAIT_FULL | (2 << 4), lim);   // the odd CTA's half
            }
            int i = 0;
            for (int t = 0; t < my_tiles && ok_run; ++t) {
                const int acc = t & 1;
                const int chunk = (unit + t * nunits) % a.nchunks;
                const uint32_t idesc = idesc_u8s8(MT, min(NC, a.cout - chunk * NC));   // chunk width
                if (!mbar_wait_w(&acce[acc], ((t >> 1) & 1) ^ 1, a.err, s_abort, ERR_WAIT_ACC | (3 << 4), lim)) break;
                tc_fence_after();
                for (int j = 0; j < NS; ++j, ++i) {
                    const int s = i % SA;
                    const int gc = min(KSTEP, G - j * KSTEP);        // K groups in this stage
                    if (!mbar_wait_w(&fullA[s], (i / SA) & 1, a.err, s_abort, ERR_WAIT_FULL | (4 << 4), lim)) { ok_run = false; break; }
                    uint32_t bbase;
                    int sbi = 0;
                    if (a.b_resident) {
                        bbase = b0 + j * KSTEP * btile;
                    } else {
                        sbi = i % a.sb;
                        if (!mbar_wait_w(&fullB[sbi], (i / a.sb) & 1, a.err, s_abort, ERR_WAIT_FULL | (5 << 4), lim)) { ok_run = false; break; }
                        bbase = b0 + sbi * bstage;
                    }
                    tc_fence_after();
                    const uint32_t abase = a0 + s * ASTAGE;
#pragma unroll
                    for (int x = 0; x < UNITS; ++x) {
                        // conv1: unit x = K group j*KSTEP + x; transition: pixel x of the squares
                        if (TRANS || x < gc) {
                            const uint64_t bd = sdesc(bbase + (TRANS ? 0 : x * btile), 16, 256, LAYOUT_SW32);
                            const uint32_t accum = (j | x) ? 1u : 0u;   // the tile's first MMA overwrites
                            if constexpr (PAIR) {
                                umma_u8s8_ts_pair_w(tmem + acc * NC, tmem + TMEM_A_COL + s * (UNITS * 8) + x * 8, bd,
                                                    idesc, accum);
                            } else if constexpr (TMEM_A) {
                                umma_u8s8_ts_w(tmem + acc * NC, tmem + TMEM_A_COL + s * (UNITS * 8) + x * 8, bd,
                                               idesc, accum);
                            } else {
                                const uint64_t ad = sdesc(abase + x * 4096, 16, 256, LAYOUT_SW32);
                                umma_u8s8_w(tmem + acc * NC, ad, bd, idesc, accum);
                            }
                        }
                    }
                    if constexpr (PAIR) {
                        umma_commit_pair_w(&emptyA[s]);
                    } else {
                        umma_commit_w(&emptyA[s]);
                        if (!a.b_resident) umma_commit_w(&emptyB[sbi]);
                    }
                }
                if (!ok_run) break;
                if constexpr (PAIR) umma_commit_pair_w(&accf[acc]);
                else umma_commit_w(&accf[acc]);
            }
            __syncwarp();
        }
    } else if (warp == 1) {
        // ---------------- store producer ----------------
        // Lane 0 waits for the slot and posts the stage's bytes; lanes 0 .. gc - 1 then each issue
        // one K group's copy (one instruction for the whole stage). Stage i uses ring slot i % SR in
        // its (i / SR)-th round, both kept as running counters (SR is a launch parameter for conv1).
        int i = 0, rs = 0, rph = 0;
        for (int t = 0; t < my_tiles; ++t) {
            const int tile = unit + t * nunits;
            const int m0 = (tile / a.nchunks) * MT + static_cast<int>(rank) * 128;
            const int cnt = min(128, rows - m0);               // pair: <= 0 past the last rows
            size_t off;
            uint32_t bytes;
            int ntl = 0;                                       // transition, tile-major: tiles of the span
            if (TRANS) {
                int first, end;
                trans_span(m0, cnt, HW, a.W, &first, &end);
                if (a.tg > 0) {
                    // whole 4 KB tiles first / 128 .. (end - 1) / 128 of each K group
                    off = static_cast<size_t>(first >> 7) * a.tg * 4096;
                    ntl = ((end - 1) >> 7) - (first >> 7) + 1;
                    bytes = static_cast<uint32_t>(ntl) * 4096u;
                } else {
                    off = static_cast<size_t>(first) * 32;
                    bytes = static_cast<uint32_t>(end - first) * 32;
                }
            } else if (a.tg > 0) {
                // tile-major: a stage is the tile's groups j*KSTEP .. in one contiguous run of 4 KB each
                // (whole 128-row tiles are allocated, so a partial last tile is copied whole)
                off = static_cast<size_t>(m0 >> 7) * a.tg * 4096;
                bytes = cnt > 0 ? 4096u : 0u;
            } else {
                off = static_cast<size_t>(m0 < rows ? m0 : 0) * 32;
                bytes = cnt > 0 ? static_cast<uint32_t>(cnt) * 32 : 0u;
            }
            bool ok_run = true;
            for (int j = 0; j < NS; ++j, ++i) {
                const int s = rs, ph = rph;
                if (++rs == SR) {
                    rs = 0;
                    rph ^= 1;
                }
                const int gc = min(KSTEP, G - j * KSTEP);
                int ok = 1;
                if (lane == 0) {
                    ok = mbar_wait(&freeR[s], ph ^ 1, a.err, s_abort, ERR_WAIT_EMPTY | (6 << 4), lim) ? 1 : 0;
                    if (ok) mbar_expect_tx(&fullR[s], bytes * gc);
                }
                if (!__shfl_sync(0xffffffffu, ok, 0)) { ok_run = false; break; }
                if (a.fault == 1 && blockIdx.x == 0 && i == 0) {
                    // test hook: stage 0 is announced but never copied, so its consumers' wait runs out
                    // (every other copy of the CTA is issued and lands long before that)
                    continue;
                }
                if (TRANS && a.tg > 0) {
                    // one 4 KB copy per tile of the span, tiles tg groups apart (two groups per copy,
                    // 8 KB contiguous, measured 19 % slower per transition on B200)
                    if (lane < ntl)
                        bulk_g2s(sR + s * RB + lane * 4096,
                                 a.in0 + off + (static_cast<size_t>(lane) * a.tg + j) * 4096, 4096u, &fullR[s]);
                } else if (!TRANS && a.tg > 0) {
                    if (lane == 0 && bytes > 0)
                        bulk_g2s(sR + s * RB, a.in0 + off + static_cast<size_t>(j) * KSTEP * 4096,
                                 static_cast<uint32_t>(gc) * 4096u, &fullR[s]);
                } else if (lane < gc && bytes > 0) {                 // one copy per K group, 4 KB apart
                    const int g = j * KSTEP + lane;
                    const int8_t* src = g < G0 ? a.in0 + g * gstride + off : a.seg + (g - G0) * gstride + off;
                    bulk_g2s(sR + s * RB + lane * (RB / KSTEP), src, bytes, &fullR[s]);
                }
            }
            if (!ok_run) break;
        }
        __syncwarp();
    } else if (warp == 2) {
        // ---------------- weight producer ----------------
        if (lane == 0 && T > 0) {
            if (PAIR && rank == 1 && a.b_resident) {
                // this CTA's weight half has landed: tell the issuing CTA
                if (mbar_wait(&fullB[0], 0, a.err, s_abort, ERR_WAIT_FULL | (7 << 4), lim)) mbar_arrive_at(&fullB[1], 0);
            }
            if (!a.b_resident) {
                int i = 0;
                for (int t = 0; t < my_tiles; ++t) {
                    const int tile = unit + t * nunits;
                    const int chunk = tile % a.nchunks;
                    const int cbt = min(NC, a.cout - chunk * NC) * 32;      // weight tile bytes of the chunk
                    const uint8_t* wc = a.wu + static_cast<size_t>(G) * 32 * chunk * NC;
                    bool ok_run = true;
                    for (int j = 0; j < NS; ++j, ++i) {
                        const int s = i % a.sb;
                        const int gc = min(KSTEP, G - j * KSTEP);
                        if (!mbar_wait(&emptyB[s], ((i / a.sb) & 1) ^ 1, a.err, s_abort, ERR_WAIT_EMPTY | (8 << 4), lim)) { ok_run = false; break; }
                        // the gc weight tiles of the stage are contiguous in the prepared table
                        mbar_expect_tx(&fullB[s], static_cast<uint32_t>(gc * cbt));
                        bulk_g2s(sB + s * bstage, wc + static_cast<size_t>(j) * KSTEP * cbt,
                                 static_cast<uint32_t>(gc * cbt), &fullB[s]);
                    }
                    if (!ok_run) break;
                }
            }
        }
        __syncwarp();
    } else if (warp <= 10 && TMEM_A) {
        // ---------------- prologue, A into TMEM (conv1) ----------------
        // Warp w writes TMEM lanes 32 (w % 4) .. + 31; the two warps of a lane quadrant alternate
        // stages. The stores use the 16x256b shape: thread t holds K bytes 8 (t % 4) .. + 7 (channels
        // 8 (t % 4) .. + 7 of each unit's K group) of rows t / 4 + {0, 8, 16, 24} of the quadrant, so
        // it needs only those 8 channels' BN pairs (two 16-byte table reads per unit) and its raw
        // reads are 8-byte rows without bank conflicts.
        const int q = warp & 3, kk = (warp - 3) >> 2;
        const int t0 = lane & 3, t1 = lane >> 2;
        const uint32_t tlane = static_cast<uint32_t>(q * 32) << 16;
        const int roff = (q * 32 + t1) * 32 + t0 * 8;     // this thread's first raw bytes in a unit
        int j = kk;                                   // stage index within the tile (i = t * NS + j)
        while (j >= NS) j -= NS;
        int rs = kk, rph = 0;                         // raw slot i % SR and round parity (i / SR) & 1
        for (int i = kk; i < T; i += 2) {
            const int s = rs, ph = rph, sa = i % SA;
            rs += 2;                                  // SR is even: the slot wraps exactly at SR
            if (rs >= SR) {
                rs -= SR;
                rph ^= 1;
            }
            const int gc = min(KSTEP, G - j * KSTEP);
            const int j_this = j;
            j += 2;
            while (j >= NS) j -= NS;
            // (the lanes of the warp poll the same barrier and abort flag in lockstep, so they leave
            // together; tcgen05.st below is warp-collective)
            if (!mbar_wait(&fullR[s], ph, a.err, s_abort, ERR_WAIT_FULL | (9 << 4), lim)) break;
            if (!mbar_wait(&emptyA[sa], ((i / SA) & 1) ^ 1, a.err, s_abort, ERR_WAIT_EMPTY | (10 << 4), lim)) break;
            tc_fence_after();
            // res[16 h + 4 x + e]: unit x (K group), rows t/4 + 16 h (e < 2) and t/4 + 16 h + 8 (e >= 2),
            // K bytes 8 (t % 4) + 4 (e & 1) .. + 3; the registers stay live until tcgen05.wait::st
            uint32_t res[32];
#pragma unroll
            for (int x = 0; x < UNITS; ++x) {
                if (x >= gc) {                                // short last stage: columns never read
#pragma unroll
                    for (int e = 0; e < 4; ++e) res[4 * x + e] = res[16 + 4 * x + e] = 0u;
                    continue;
                }
                const int g = j_this * KSTEP + x;
                const uint8_t* src = sR + s * RB + x * 4096 + roff;
                const uint2 r0 = *reinterpret_cast<const uint2*>(src);            // row t/4
                const uint2 r1 = *reinterpret_cast<const uint2*>(src + 8 * 32);   // row t/4 + 8
                const uint2 r2 = *reinterpret_cast<const uint2*>(src + 16 * 32);  // row t/4 + 16
                const uint2 r3 = *reinterpret_cast<const uint2*>(src + 24 * 32);  // row t/4 + 24
                if (F16) {
                    const uint4* tb = reinterpret_cast<const uint4*>(sTab + g * 128) + 2 * t0;
                    const uint4 ta = tb[0], tc = tb[1];          // channels 8 t0 .. + 3, + 4 .. + 7
                    res[4 * x + 0] = prologue_f16x4_ob(r0.x ^ XM, ta.x, ta.y, ta.z, ta.w);
                    res[4 * x + 1] = prologue_f16x4_ob(r0.y ^ XM, tc.x, tc.y, tc.z, tc.w);
                    res[4 * x + 2] = prologue_f16x4_ob(r1.x ^ XM, ta.x, ta.y, ta.z, ta.w);
                    res[4 * x + 3] = prologue_f16x4_ob(r1.y ^ XM, tc.x, tc.y, tc.z, tc.w);
                    res[16 + 4 * x + 0] = prologue_f16x4_ob(r2.x ^ XM, ta.x, ta.y, ta.z, ta.w);
                    res[16 + 4 * x + 1] = prologue_f16x4_ob(r2.y ^ XM, tc.x, tc.y, tc.z, tc.w);
                    res[16 + 4 * x + 2] = prologue_f16x4_ob(r3.x ^ XM, ta.x, ta.y, ta.z, ta.w);
                    res[16 + 4 * x + 3] = prologue_f16x4_ob(r3.y ^ XM, tc.x, tc.y, tc.z, tc.w);
                } else {
                    const float2* tb = reinterpret_cast<const float2*>(sTab) + g * 32 + 8 * t0;
                    res[4 * x + 0] = prologue_f32x4_ob(r0.x ^ XM, tb);
                    res[4 * x + 1] = prologue_f32x4_ob(r0.y ^ XM, tb + 4);
                    res[4 * x + 2] = prologue_f32x4_ob(r1.x ^ XM, tb);
                    res[4 * x + 3] = prologue_f32x4_ob(r1.y ^ XM, tb + 4);
                    res[16 + 4 * x + 0] = prologue_f32x4_ob(r2.x ^ XM, tb);
                    res[16 + 4 * x + 1] = prologue_f32x4_ob(r2.y ^ XM, tb + 4);
                    res[16 + 4 * x + 2] = prologue_f32x4_ob(r3.x ^ XM, tb);
                    res[16 + 4 * x + 3] = prologue_f32x4_ob(r3.y ^ XM, tb + 4);
                }
            }
            tmem_st16x256_2x4(tmem + tlane + TMEM_A_COL + sa * (UNITS * 8), res);
            __syncwarp();
            if (lane == 0) mbar_arrive(&freeR[s]);
            tmem_wait_st(res);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                if constexpr (PAIR) mbar_arrive_at(&fullA[sa], 0);      // the issuing CTA's barrier
                else mbar_arrive(&fullA[sa]);
            }
        }
    } else if (warp <= 10) {
        // ---------------- prologue ----------------
        // One warp owns a whole unit (128 rows x 32 B = 256 chunks of 16 B; chunk c = jj * 32 + lane is
        // row c / 2, half c % 2), so every shared-memory access of the warp is 512 contiguous bytes;
        // the 8 warps work on two stages at once.
        const int pw = warp - 3;
        const int h = lane & 1;
        const int W = a.W, W2 = W >> 1;
        // warp pw always holds unit x = pw % 4 of the stages i = pw / 4, + 2, ...; the shared-memory
        // offsets of its rows depend only on the tile, so they are computed once per tile, and the
        // stage's tile t and K group j advance as running counters (i = t * NS + j)
        const int x = pw & 3;
        int t = 0, j = pw >> 2;
        while (j >= NS) {
            j -= NS;
            ++t;
        }
        int off[8];
        int t_off = -1;
        for (int i = pw >> 2; i < T; i += 2) {
            if (t != t_off) {
                t_off = t;
                if (TRANS) {
                    // pooled pixel m0 + r -> global pooled row gr (= n * H/2 + oy) and column ox; its
                    // input pixel (2 oy + dy, 2 ox + dx) sits 2W (gr - gr0) + dy W + 2 ox + dx pixels after
                    // the first pixel of the copied span
                    const int tile = unit + t * nunits;
                    const int m0 = (tile / a.nchunks) * 128;
                    const int gr0 = m0 / W2;
                    const int first = 2 * W * gr0;                // first input pixel of the copied span
                    int m = min(m0 + (lane >> 1), rows - 1);
                    int gr = m / W2, ox = m - gr * W2;
#pragma unroll
                    for (int jj = 0; jj < 8; ++jj) {
                        const int rel = 2 * W * (gr - gr0) + (x >> 1) * W + 2 * ox + (x & 1);
                        if (a.tg > 0) {                           // tile-major span: whole 4 KB tiles
                            const int q = first + rel;
                            off[jj] = ((q >> 7) - (first >> 7)) * 4096 + (q & 127) * 32 + h * 16;
                        } else {
                            off[jj] = rel * 32 + h * 16;
                        }
                        if (jj < 7) {                             // next chunk row: +16 pooled pixels
                            const int step = min(16, rows - 1 - m);
                            m += step;
                            ox += step;
                            while (ox >= W2) { ox -= W2; ++gr; }
                        }
                    }
                } else {
#pragma unroll
                    for (int jj = 0; jj < 8; ++jj) off[jj] = x * 4096 + (jj * 32 + lane) * 16;
                }
            }
            const int s = i % SR, sa = i % SA;
            const int gc = min(KSTEP, G - j * KSTEP);
            const bool active = TRANS || x < gc;                  // conv1: the tile's last stage may be short
            const int g = TRANS ? j : j * KSTEP + x;              // K group of this unit
            j += 2;                                               // the next stage of this warp (NS >= 2)
            while (j >= NS) {
                j -= NS;
                ++t;
            }
            if (!mbar_wait(&fullR[s], (i / SR) & 1, a.err, s_abort, ERR_WAIT_FULL | (11 << 4), lim)) break;
            uint4 q[8];
            if (active) {
#pragma unroll
                for (int jj = 0; jj < 8; ++jj) q[jj] = *reinterpret_cast<const uint4*>(sR + s * RB + off[jj]);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&freeR[s]);
            uint4 res[8];
            if (active) {
                if (F16) {
                    const uint4* tb = reinterpret_cast<const uint4*>(sTab + (g * 16 + h * 8) * 8);
                    const uint4 t0 = tb[0], t1 = tb[1], t2 = tb[2], t3 = tb[3];    // 8 channel pairs (A, B)
#pragma unroll
                    for (int jj = 0; jj < 8; ++jj) {
                        res[jj].x = prologue_f16x4_ob(q[jj].x ^ XM, t0.x, t0.y, t0.z, t0.w);
                        res[jj].y = prologue_f16x4_ob(q[jj].y ^ XM, t1.x, t1.y, t1.z, t1.w);
                        res[jj].z = prologue_f16x4_ob(q[jj].z ^ XM, t2.x, t2.y, t2.z, t2.w);
                        res[jj].w = prologue_f16x4_ob(q[jj].w ^ XM, t3.x, t3.y, t3.z, t3.w);
                    }
                } else {
                    const float2* tb = reinterpret_cast<const float2*>(sTab) + g * 32 + h * 16;
#pragma unroll
                    for (int jj = 0; jj < 8; ++jj) {
                        res[jj].x = prologue_f32x4_ob(q[jj].x ^ XM, tb);
                        res[jj].y = prologue_f32x4_ob(q[jj].y ^ XM, tb + 4);
                        res[jj].z = prologue_f32x4_ob(q[jj].z ^ XM, tb + 8);
                        res[jj].w = prologue_f32x4_ob(q[jj].w ^ XM, tb + 12);
                    }
                }
            }
            if (!mbar_wait(&emptyA[sa], ((i / SA) & 1) ^ 1, a.err, s_abort, ERR_WAIT_EMPTY | (12 << 4), lim)) break;
            if (active) {
                uint8_t* dst = sA + sa * ASTAGE + x * 4096;
#pragma unroll
                for (int jj = 0; jj < 8; ++jj) {
                    const int r = (jj * 32 + lane) >> 1;
                    *reinterpret_cast<uint4*>(dst + r * 32 + ((h ^ ((r >> 2) & 1)) << 4)) = res[jj];
                }
                fence_async_smem();
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&fullA[sa]);
        }
    } else {
        // ---------------- epilogue ----------------
        // TMEM accumulators hold the int32 sums (each tile's first MMA overwrites); the int -> float
        // conversion is an integer add of the MAGIC bits and one float subtraction (one packed f32x2
        // subtraction per channel pair; conv1's 255 v + 2^23 is one packed fma per pair as well).
        const int quad = warp & 3, half = (warp - 11) >> 2;
        const float4* gd4 = reinterpret_cast<const float4*>(sGd);
        // transition: the rounding add whose low byte is q (1.5 * 2^23), or q + 128 for a tile-major
        // output store (offset binary; the added 128 keeps the sum even, so ties still round to even q)
        const float omag = a.tg_out > 0 ? 12583040.0f : 12582912.0f;
        // the conversion mode is fixed per launch: one instantiation of the tile loop per mode
        auto tiles = [&](auto fast_tag) {
            constexpr bool FAST = decltype(fast_tag)::value;
            for (int t = 0; t < my_tiles; ++t) {
                const int acc = t & 1;
                if (!mbar_wait(&accf[acc], (t >> 1) & 1, a.err, s_abort, ERR_WAIT_ACC | (13 << 4), lim)) break;
                tc_fence_after();
                const int tile = unit + t * nunits;
                const int nch = TRANS ? a.nchunks : 1;                   // conv1: one chunk
                const int chunk = tile % nch;
                const int ncol = min(NC, a.cout - chunk * NC) >> 1;      // columns of this warp
                const int m = (tile / nch) * MT + static_cast<int>(rank) * 128 + quad * 32 + lane;
                const uint32_t taddr = tmem + (static_cast<uint32_t>(quad * 32) << 16) + acc * NC + half * ncol;
                // requantise 16 columns (output channels c0 ..) of this warp's 32 rows and store them
                auto finish = [&](const uint32_t (&v)[16], int cb) {
                    const int c0 = chunk * NC + half * ncol + cb;      // first output channel (even)
                    const float4* gdp = gd4 + (c0 >> 1);               // (g, d) pairs of channels c0 ..
                    uint32_t wd[4];
    #pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        uint32_t b[4];
    #pragma unroll
                        for (int e = 0; e < 2; ++e) {
                            const int c = 4 * j + 2 * e;
                            float2 f;
                            if constexpr (FAST) {
                                f = __fadd2_rn(make_float2(__uint_as_float(v[c] + ACC_MAGIC), __uint_as_float(v[c + 1] + ACC_MAGIC)),
                                               make_float2(-ACC_MAGIC_F, -ACC_MAGIC_F));
                            } else {
                                f = make_float2(__int2float_rn(static_cast<int32_t>(v[c])),
                                                __int2float_rn(static_cast<int32_t>(v[c + 1])));
                            }
                            const float4 p = gdp[c >> 1];   // transition: (g0, d0, g1, d1); conv1: (g0, g1, d0, d1)
                            float2 r;
                            if (TRANS) {
                                r.x = fminf(fmaxf(p.x * f.x, -127.0f), 127.0f) + omag;
                                r.y = fminf(fmaxf(p.z * f.y, -127.0f), 127.0f) + omag;
                            } else {
                                // sat(g acc + d) per channel (one rounding each), then 255 v + 2^23 on the pair
                                r = __ffma2_rn(make_float2(__saturatef(fmaf(p.x, f.x, p.z)), __saturatef(fmaf(p.y, f.y, p.w))),
                                               make_float2(255.0f, 255.0f), make_float2(8388608.0f, 8388608.0f));
                            }
                            b[2 * e] = __float_as_uint(r.x);
                            b[2 * e + 1] = __float_as_uint(r.y);
                        }
                        wd[j] = __byte_perm(__byte_perm(b[0], b[1], 0x0040), __byte_perm(b[2], b[3], 0x0040), 0x5410);
                    }
                    if (m < rows) {
                        uint8_t* o = static_cast<uint8_t*>(a.out);
                        // transition: next block input, group-major [c_out / 32][N * HW / 4][32] or groups
                        // 0 .. c_out / 32 - 1 of its tile-major store; conv1: bottleneck planes of 16
                        // channels [8][N * HW][16]
                        size_t off;
                        if (TRANS && a.tg_out > 0)
                            off = ((static_cast<size_t>(m >> 7) * a.tg_out + (c0 >> 5)) << 12) + (m & 127) * 32 + (c0 & 16);
                        else if (TRANS)
                            off = (static_cast<size_t>(c0 >> 5) * rows + m) * 32 + (c0 & 16);
                        else
                            off = (static_cast<size_t>(c0 >> 4) * rows + m) * 16;
                        *reinterpret_cast<uint4*>(o + off) = make_uint4(wd[0], wd[1], wd[2], wd[3]);
                    }
                };
                // 16-column chunks, each chunk's TMEM load issued one chunk ahead (tcgen05.wait::ld waits
                // for every earlier load, so the load of chunk k + 1 is in flight while chunk k is worked)
                uint32_t va[16], vb[16];
                tmem_ld16(taddr, va);
                for (int cb = 0; cb < ncol; cb += 32) {
                    tmem_wait_ld(va);
                    tmem_ld16(taddr + cb + 16, vb);
                    finish(va, cb);
                    tmem_wait_ld(vb);
                    if (cb + 32 < ncol) tmem_ld16(taddr + cb + 32, va);
                    finish(vb, cb + 16);
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) {
                    if constexpr (PAIR) mbar_arrive_at(&acce[acc], 0);      // the issuing CTA's barrier
                    else mbar_arrive(&acce[acc]);
                }
            }
        };
        if (fast_cvt) tiles(std::true_type{});
        else tiles(std::false_type{});
    }

    tc_fence_before();
    __syncthreads();
    if constexpr (PAIR) {
        // Every MMA has completed (the epilogue saw the last accumulator), but the issuing CTA's last
        // commit arrivals on emptyA may still be landing here: wait for each barrier's final phase
        // before the CTA can exit. Then both CTAs meet, so no arrival or MMA of the pair is in flight.
        if (threadIdx.x == 0) {
            for (int sl = 0; sl < SA && sl < T; ++sl) {
                const int il = sl + SA * ((T - 1 - sl) / SA);          // last stage on barrier sl
                if (!mbar_wait(&emptyA[sl], (il / SA) & 1, a.err, s_abort, ERR_WAIT_EMPTY | (14 << 4), lim)) break;
            }
        }
        cluster_sync();
    }
    if (warp == 0) {
        tc_fence_after();
        if constexpr (PAIR) tmem_free_pair(tmem, tcols);
        else tmem_free(tmem, tcols);
    }
}

// Clusters of two that can be resident at once (both SMs of a pair free), per device.
static int pair_slots(int sms) {
    static std::atomic<int> cache[DN8_MAX_DEVICES];     // 0 = not looked up yet (threads may race to fill it)
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= DN8_MAX_DEVICES) return sms / 2;
    if (const int c = cache[dev].load(std::memory_order_relaxed); c > 0) return c;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(sms & ~1));
    cfg.blockDim = dim3(GM_THREADS);
    cfg.dynamicSmemBytes = SMEM_BUDGET + 1024;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = 2;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaFuncSetAttribute(gemm_kernel<true, false, true, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             SMEM_BUDGET + 1024) != cudaSuccess ||
        cudaOccupancyMaxActiveClusters(&n, gemm_kernel<true, false, true, true>, &cfg) != cudaSuccess || n <= 0) {
        (void)cudaGetLastError();
        n = sms / 2;
    }
    n = n < sms / 2 ? n : sms / 2;
    cache[dev].store(n, std::memory_order_relaxed);
    return n;
}

// conv1 runs on single CTAs while its weights fit resident next to the raw ring, else on CTA pairs
// (half the weights per CTA, resident for every layer of the network). Measured on B200 (same box):
// single CTAs are 5-12 % faster where both fit; pairs are 8-10 % faster than single CTAs that stream
// their weights.
template <bool F16, bool TRANS, bool OB>
static cudaError_t launch_gemm_ob(GemmArgs g, int sms, cudaStream_t st, bool pdl) {
    bool pair = false;
    size_t smem = gemm_layout(TRANS, false, g.G, g.nc, g.nchunks, g.raw_bytes, &g.sb, &g.b_resident, &g.sr) + 1024;
    if (!TRANS && !g.b_resident) {
        pair = true;
        smem = gemm_layout(TRANS, true, g.G, g.nc, g.nchunks, g.raw_bytes, &g.sb, &g.b_resident, &g.sr) + 1024;
        if (!g.b_resident) return cudaErrorInvalidConfiguration;
    }
    if (smem > 227 * 1024 || g.sb < 2) return cudaErrorInvalidConfiguration;
    const int mt = pair ? 256 : 128;
    const int ntiles = ((g.rows + mt - 1) / mt) * g.nchunks;
    if (ntiles <= 0) return cudaSuccess;
    if (!pair) {
        cudaError_t e = cudaFuncSetAttribute(gemm_kernel<F16, TRANS, false, OB>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (e != cudaSuccess) return e;
        const int grid = ntiles < sms ? ntiles : sms;
        return launch_pdl(pdl, gemm_kernel<F16, TRANS, false, OB>, dim3(grid), dim3(GM_THREADS), smem, st, g);
    }
    if constexpr (!TRANS) {
        cudaError_t e = cudaFuncSetAttribute(gemm_kernel<F16, false, true, OB>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (e != cudaSuccess) return e;
        const int slots = pair_slots(sms);
        const int pairs = ntiles < slots ? ntiles : slots;
        return launch_pdl_pairs(pdl, gemm_kernel<F16, false, true, OB>, dim3(2 * pairs), dim3(GM_THREADS), smem, st, g);
    }
    return cudaErrorInvalidConfiguration;
}
// a tile-major input store is offset binary (OB), group-major planes are signed
template <bool F16, bool TRANS>
static cudaError_t launch_gemm(const GemmArgs& g, int sms, cudaStream_t st, bool pdl) {
    return g.tg > 0 ? launch_gemm_ob<F16, TRANS, true>(g, sms, st, pdl) : launch_gemm_ob<F16, TRANS, false>(g, sms, st, pdl);
}

// conv1 keeps every layer's weights resident: on single CTAs up to 37 K groups, on CTA pairs up to 70.
bool conv1_supported(int G) {
    int sb = 0, resident = 0, sr = 0;
    const size_t smem = gemm_layout(false, true, G, 128, 1, 4 * 4096, &sb, &resident, &sr) + 1024;
    return resident && smem <= 227 * 1024;
}

// dn8_test_inject_wait_fault: armed by the test hook, consumed by the next conv1 launch of the process.
static std::atomic<int> g_fault_next{0};
static std::atomic<long long> g_limit_next{0};

void arm_wait_fault(int fault, long long wait_limit) {
    g_limit_next.store(wait_limit, std::memory_order_relaxed);
    g_fault_next.store(fault, std::memory_order_release);
}

cudaError_t launch_conv1(const dn8_conv1_args& a, int sms, cudaStream_t st, bool pdl) {
    GemmArgs g{};
    g.wait_limit = WAIT_LIMIT;
    if (const int f = g_fault_next.exchange(0, std::memory_order_acquire); f != 0) {
        g.fault = f;
        const long long lim = g_limit_next.load(std::memory_order_relaxed);
        g.wait_limit = lim > 0 ? lim : WAIT_LIMIT;
    }
    g.in0 = a.in0; g.seg = a.seg; g.wu = reinterpret_cast<const uint8_t*>(a.w); g.ab = a.ab; g.gd = a.gd;
    g.out = a.out; g.err = a.err;
    g.G0 = a.G0; g.G = a.G; g.N = a.N; g.HW = a.HW; g.W = 0;
    g.rows = a.N * a.HW; g.cout = 128; g.nc = 128; g.nchunks = 1;
    g.raw_bytes = 4 * 4096;
    g.tg = a.tile_groups;
    return a.prologue_f16 ? launch_gemm<true, false>(g, sms, st, pdl) : launch_gemm<false, false>(g, sms, st, pdl);
}

// output channels per CTA tile: 256 (TMEM: 2 x 256 columns; the last chunk of a c_out that is an
// odd multiple of 128 has 128), or 128 when c_out is 128
int trans_chunk(int cout) { return cout >= 256 ? 256 : 128; }

// Largest raw span of a transition tile: its 128 consecutive pooled pixels cover at most
// 128 / W2 pooled rows when W2 divides 128 (tiles start on a row), else ceil(128 / W2) + 1;
// each pooled row needs two whole input rows.
// tiled: whole 4 KB tiles; a span of 2 prow W pixels starting anywhere covers at most span / 128 + 2
// of them, exactly span / 128 when it starts on a tile (W / 2 divides 128: every block at 512 px).
static int trans_raw_bytes(int W, bool tiled) {
    const int W2 = W / 2;
    const int prow = (128 % W2 == 0) ? 128 / W2 : (128 + W2 - 1) / W2 + 1;
    if (tiled) {
        const int span = 2 * prow * W;
        return (128 % W2 == 0 && span % 128 == 0 ? span / 128 : span / 128 + 2) * 4096;
    }
    return ((2 * prow * W * 32 + 1023) / 1024) * 1024;
}

cudaError_t launch_trans(const dn8_trans_args& a, int sms, cudaStream_t st, bool pdl) {
    GemmArgs g{};
    g.wait_limit = WAIT_LIMIT;
    const int cout = a.G * 16;
    g.in0 = a.in0; g.seg = a.seg; g.wu = reinterpret_cast<const uint8_t*>(a.w); g.ab = a.ab; g.gd = a.gd;
    g.out = a.out; g.err = a.err;
    g.G0 = a.G0; g.G = a.G; g.N = a.N; g.HW = a.H * a.W; g.W = a.W;
    g.rows = a.N * (a.H / 2) * (a.W / 2); g.cout = cout; g.nc = trans_chunk(cout);
    g.nchunks = (cout + g.nc - 1) / g.nc;
    g.raw_bytes = trans_raw_bytes(a.W, a.tile_groups > 0);
    g.tg = a.tile_groups;
    g.tg_out = a.out_tile_groups;
    return a.prologue_f16 ? launch_gemm<true, true>(g, sms, st, pdl) : launch_gemm<false, true>(g, sms, st, pdl);
}

}  // namespace dn8
