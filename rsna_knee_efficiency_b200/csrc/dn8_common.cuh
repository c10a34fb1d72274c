// dn8_common.cuh -- device helpers shared by the sm_100a kernels of the INT8 DenseNet169 encoder:
// mbarriers with bounded waits, bulk / tensor copies, tcgen05 (TMEM allocation, kind::i8 MMA,
// commit, TMEM loads, fences), UMMA descriptors and the bit-exact prologue arithmetic.
#pragma once
#include <cstdint>
#include <cstring>
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#define DN8_DEV __device__ __forceinline__

namespace dn8 {

// ---- error reporting ------------------------------------------------------------------------
// Every wait is bounded. A wait that gives up writes its code into the launch's error word (the
// first code wins) and raises the CTA's abort flag, after which every role leaves its loop; the
// kernel still frees its TMEM and returns, so the context stays usable.
enum : int {
    ERR_NONE = 0,
    ERR_WAIT_FULL = 1,      // a consumer waited too long for a filled stage
    ERR_WAIT_EMPTY = 2,     // a producer waited too long for a free stage
    ERR_WAIT_ACC = 3,       // MMA / epilogue accumulator hand-off
    ERR_SHAPE = 4,          // launch arguments outside what the kernel supports
};
// A kernel may add the wait site in bits 4-11 (code = kind | site << 4), so that a device error
// names the barrier that ran out.
// ~2^32 SM cycles (about 2 s at 2 GHz): far beyond any legitimate wait of these kernels.
constexpr long long WAIT_LIMIT = 1ll << 32;

DN8_DEV uint32_t smem_u32(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

DN8_DEV void raise_error(int* err, volatile int* abort_flag, int code) {
    if (err) atomicCAS(err, 0, code);
    *abort_flag = 1;
}

// ---- mbarrier -------------------------------------------------------------------------------
DN8_DEV void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
DN8_DEV void mbar_fence_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
DN8_DEV void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
DN8_DEV void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;"
                 ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
DN8_DEV bool mbar_try(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
                 "selp.u32 %0, 1, 0, p;\n\t}"
                 : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity) : "memory");
    return ok != 0;
}
// As mbar_try, but a thread whose phase is not complete is suspended until it completes or about
// `ns` nanoseconds pass, so a waiting warp issues almost no instructions while it waits.
DN8_DEV bool mbar_try_sleep(uint64_t* bar, uint32_t parity, uint32_t ns) {
    uint32_t ok;
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2, %3;\n\t"
                 "selp.u32 %0, 1, 0, p;\n\t}"
                 : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity), "r"(ns) : "memory");
    return ok != 0;
}
// Waits for the phase of parity `parity` to complete. Returns false (error raised) on timeout (after
// `limit` SM cycles) or when another role has already aborted.
DN8_DEV bool mbar_wait(uint64_t* bar, uint32_t parity, int* err, volatile int* abort_flag, int code,
                       long long limit = WAIT_LIMIT) {
    if (mbar_try(bar, parity)) return true;
    const long long t0 = clock64();
    while (!mbar_try_sleep(bar, parity, 100000u)) {
        if (*abort_flag) return false;
        if (clock64() - t0 > limit) {
            raise_error(err, abort_flag, code);
            return false;
        }
    }
    return true;
}

// ---- programmatic dependent launch -----------------------------------------------------------
// Kernels are launched with programmatic stream serialization: the next kernel of the stream may
// start (and do its setup: barriers, TMEM, constant tables) while this one finishes. Every kernel
// lets its dependents launch once its own setup is done, then waits for its predecessor's
// completion (and memory) before it reads activations or writes any output.
DN8_DEV void griddep_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
DN8_DEV void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// ---- bulk copies / TMA ----------------------------------------------------------------------
// Contiguous global -> shared copy (16-byte aligned, size a multiple of 16), completing on `bar`.
DN8_DEV void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar)) : "memory");
}
// 4-D tiled tensor load into this CTA's shared memory, completing on `bar`.
DN8_DEV void tma_load_4d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1, int c2, int c3) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3, %4, %5}], [%6];"
        ::"r"(smem_u32(dst)), "l"(map), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_u32(bar))
        : "memory");
}
DN8_DEV void prefetch_tensormap(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}
// Generic-proxy shared-memory writes made visible to the async proxy (tensor core, TMA).
DN8_DEV void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// ---- tcgen05 --------------------------------------------------------------------------------
// One full warp allocates; the base address is written to shared memory.
DN8_DEV void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                 ::"r"(smem_u32(dst_smem)), "r"(ncols) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
DN8_DEV void tmem_free(uint32_t base, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(base), "r"(ncols) : "memory");
}
DN8_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
DN8_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Shared-memory matrix descriptor (sm_100 "version 1"): start, leading / stride byte offsets.
enum : uint32_t { LAYOUT_NONE = 0, LAYOUT_SW32 = 6 };
DN8_DEV uint64_t sdesc(uint32_t saddr, uint32_t lbo, uint32_t sbo, uint32_t layout) {
    return static_cast<uint64_t>((saddr >> 4) & 0x3FFFu) |
           (static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16) |
           (static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46) |
           (static_cast<uint64_t>(layout) << 61);
}
// Instruction descriptor of tcgen05.mma kind::i8: D s32, A u8, B s8, both K-major.
constexpr uint32_t idesc_u8s8(int M, int N) {
    return (2u << 4) | (0u << 7) | (1u << 10) | (static_cast<uint32_t>(N >> 3) << 17) |
           (static_cast<uint32_t>(M >> 4) << 24);
}
// ---- warp-converged MMA issue -----------------------------------------------------------------
// The MMA role runs as one whole, converged warp: its control flow and operands are warp-uniform and
// elect.sync picks the issuing lane (the lowest active one, so MMAs and their commits come from the
// same thread) inside each asm. A lane-0-only issuer (a divergent branch) measured ~116 SM clocks per
// M128 x N x K32 kind::i8 MMA on B200 for every N <= 128; the converged warp issues one every ~79
// clocks at N = 128 (the tensor rate is 64).
DN8_DEV void umma_u8s8_w(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
    asm volatile("{\n\t.reg .pred p, e;\n\t.reg .b32 l;\n\t"
                 "setp.ne.b32 p, %4, 0;\n\t"
                 "elect.sync l|e, 0xffffffff;\n\t"
                 "@e tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}"
                 ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate) : "memory");
}
// A from TMEM: M = 128 rows x K = 32 bytes in 8 consecutive TMEM columns, row m in lane m, bytes
// 4c .. 4c+3 of the row in column c.
DN8_DEV void umma_u8s8_ts_w(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
    asm volatile("{\n\t.reg .pred p, e;\n\t.reg .b32 l;\n\t"
                 "setp.ne.b32 p, %4, 0;\n\t"
                 "elect.sync l|e, 0xffffffff;\n\t"
                 "@e tcgen05.mma.cta_group::1.kind::i8 [%0], [%1], %2, %3, p;\n\t}"
                 ::"r"(tmem_d), "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate) : "memory");
}
DN8_DEV void umma_commit_w(uint64_t* bar) {
    asm volatile("{\n\t.reg .pred e;\n\t.reg .b32 l;\n\t"
                 "elect.sync l|e, 0xffffffff;\n\t"
                 "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}"
                 ::"r"(smem_u32(bar)) : "memory");
}
// ---- CTA pairs (clusters of two; tcgen05 cta_group::2) -------------------------------------------
// The even CTA of a pair issues M = 256 MMAs whose A rows 0-127 / 128-255 and B rows (output
// channels) 0-63 / 64-127 live in CTA 0 / CTA 1 at the same TMEM / shared-memory offsets; each CTA's
// TMEM receives its own 128 accumulator rows. A CTA signals the other one by arriving on the barrier
// at the same offset in its shared memory; the data it hands over is in TMEM (ordered by the tcgen05
// waits and fences around the arrive) or was written by the async proxy, so the arrive needs no
// cluster-scope release (which would also wait for the thread's global stores).
DN8_DEV uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
// All threads of both CTAs (also a CTA-wide barrier).
DN8_DEV void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Arrives on the barrier at the same shared-memory offset in CTA `rank` of the cluster.
DN8_DEV void mbar_arrive_at(uint64_t* bar, uint32_t rank) {
    asm volatile("{\n\t.reg .b32 ra;\n\t"
                 "mapa.shared::cluster.u32 ra, %0, %1;\n\t"
                 "mbarrier.arrive.shared::cluster.b64 _, [ra];\n\t}"
                 ::"r"(smem_u32(bar)), "r"(rank) : "memory");
}
// A float of CTA `rank`'s shared memory at the offset of `p` in this CTA (distributed shared memory).
DN8_DEV float ld_peer_f32(const float* p, uint32_t rank) {
    float v;
    asm volatile("{\n\t.reg .b32 ra;\n\t"
                 "mapa.shared::cluster.u32 ra, %1, %2;\n\t"
                 "ld.shared::cluster.f32 %0, [ra];\n\t}"
                 : "=f"(v) : "r"(smem_u32(p)), "r"(rank) : "memory");
    return v;
}
// One full warp of EACH CTA of the pair (the same warp) allocates; both get the same base address.
DN8_DEV void tmem_alloc_pair(uint32_t* dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;"
                 ::"r"(smem_u32(dst_smem)), "r"(ncols) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
DN8_DEV void tmem_free_pair(uint32_t base, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(base), "r"(ncols) : "memory");
}
// D (+)= A[tmem] * B[smem]^T over both CTAs of the pair (M = 256), issued from the even CTA by a
// converged warp (one elected lane).
DN8_DEV void umma_u8s8_ts_pair_w(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                                 uint32_t accumulate) {
    asm volatile("{\n\t.reg .pred p, e;\n\t.reg .b32 l;\n\t"
                 "setp.ne.b32 p, %4, 0;\n\t"
                 "elect.sync l|e, 0xffffffff;\n\t"
                 "@e tcgen05.mma.cta_group::2.kind::i8 [%0], [%1], %2, %3, {%5, %5, %5, %5, %5, %5, %5, %5}, p;\n\t}"
                 ::"r"(tmem_d), "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(0u) : "memory");
}
// Arrives once on `bar` in BOTH CTAs of the pair when the pair MMAs issued so far have completed.
DN8_DEV void umma_commit_pair_w(uint64_t* bar) {
    asm volatile("{\n\t.reg .pred e;\n\t.reg .b32 l;\n\t"
                 "elect.sync l|e, 0xffffffff;\n\t"
                 "@e tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;\n\t}"
                 ::"r"(smem_u32(bar)), "h"(static_cast<uint16_t>(3)) : "memory");
}
// Every lane waits; the warp continues only if all of them saw the phase (a timeout or an abort seen
// by any lane stops the whole warp, so the issuing loop stays converged).
DN8_DEV bool mbar_wait_w(uint64_t* bar, uint32_t parity, int* err, volatile int* abort_flag, int code,
                         long long limit = WAIT_LIMIT) {
    return __all_sync(0xffffffffu, mbar_wait(bar, parity, err, abort_flag, code, limit)) != 0;
}
// tcgen05.ld writes its registers asynchronously: their values may be read only after
// tcgen05.wait::ld. A wait with a "memory" clobber alone orders memory, not registers, so the compiler
// could schedule arithmetic on the loaded registers above it. The waits below name the registers of
// the outstanding loads as in/out operands, so every use depends on the wait; reg_bind extends that
// to more registers after a wait (an empty asm, ordered after the wait as both are volatile).
#define DN8_B8(i) "+r"(r[i]), "+r"(r[i + 1]), "+r"(r[i + 2]), "+r"(r[i + 3]), \
                  "+r"(r[i + 4]), "+r"(r[i + 5]), "+r"(r[i + 6]), "+r"(r[i + 7])
DN8_DEV void tmem_wait_ld(uint32_t (&r)[16]) {
    asm volatile("tcgen05.wait::ld.sync.aligned;" : DN8_B8(0), DN8_B8(8) : : "memory");
}
DN8_DEV void tmem_wait_ld(uint32_t (&r)[32]) {
    asm volatile("tcgen05.wait::ld.sync.aligned;" : DN8_B8(0), DN8_B8(8), DN8_B8(16), DN8_B8(24) : : "memory");
}
DN8_DEV void reg_bind(uint32_t (&r)[16]) { asm volatile("" : DN8_B8(0), DN8_B8(8) : : "memory"); }
DN8_DEV void reg_bind(uint32_t (&r)[32]) {
    asm volatile("" : DN8_B8(0), DN8_B8(8), DN8_B8(16), DN8_B8(24) : : "memory");
}
#undef DN8_B8

#define DN8_R8(i) "=r"(r[i]), "=r"(r[i + 1]), "=r"(r[i + 2]), "=r"(r[i + 3]), \
                  "=r"(r[i + 4]), "=r"(r[i + 5]), "=r"(r[i + 6]), "=r"(r[i + 7])
// 32 lanes x 32 consecutive 32-bit columns: thread t of the warp gets row (lane base + t).
DN8_DEV void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x32.b32 "
                 "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
                 "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
                 : DN8_R8(0), DN8_R8(8), DN8_R8(16), DN8_R8(24)
                 : "r"(taddr) : "memory");
}
DN8_DEV void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x16.b32 "
                 "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
                 : DN8_R8(0), DN8_R8(8)
                 : "r"(taddr) : "memory");
}
// 32 lanes x 32 columns as two 16x256b.x4 stores (lanes +0 and +16 of the warp's quadrant):
// thread t's registers 4k .. 4k+3 are (row t/4, columns 8k + 2(t%4), 8k + 2(t%4) + 1) and the same
// columns of row t/4 + 8; r[0..15] go to the first 16 lanes, r[16..31] to the next 16.
DN8_DEV void tmem_st16x256_2x4(uint32_t taddr, const uint32_t (&r)[32]) {
    asm volatile("tcgen05.st.sync.aligned.16x256b.x4.b32 [%0], "
                 "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};"
                 ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]),
                   "r"(r[7]), "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
                   "r"(r[15])
                 : "memory");
    asm volatile("tcgen05.st.sync.aligned.16x256b.x4.b32 [%0], "
                 "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};"
                 ::"r"(taddr + (16u << 16)), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]),
                   "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
                   "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
                 : "memory");
}
DN8_DEV void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
// tcgen05.st reads its source registers asynchronously: they must keep their values until
// tcgen05.wait::st. This wait names them as inputs, so the compiler keeps them live (and does not
// reuse them) until the stores have completed.
DN8_DEV void tmem_wait_st(const uint32_t (&r)[32]) {
    asm volatile("tcgen05.wait::st.sync.aligned;"
                 ::"r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
                   "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]),
                   "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]),
                   "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
                 : "memory");
}
#undef DN8_R8

// ACC_MAGIC = the bits of the float 1.5 * 2^23: the int32 MAGIC + acc (an accumulator armed with MAGIC,
// or an integer add) read as a float is 1.5 * 2^23 + acc exactly while |acc| < 2^22, so (float)acc
// is one subtraction.
constexpr uint32_t ACC_MAGIC = 0x4B400000u;
constexpr float ACC_MAGIC_F = 12582912.0f;

// ---- packed fp32 pairs (sm_100 f32x2) --------------------------------------------------------
// Packed fp32 pairs (one f32x2 instruction for two lanes' worth of fp32 math, each element rounded
// exactly as the scalar operation).
DN8_DEV float2 f2_pack(float a, float b) { return make_float2(a, b); }
DN8_DEV void f2_unpack(float2 r, float& a, float& b) {
    a = r.x;
    b = r.y;
}
DN8_DEV float2 f2_fma(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }

// ---- bit-exact prologue / epilogue arithmetic -----------------------------------------------
// fp16 prologue of 4 store bytes (channels c..c+3, c even): u = rint(255 * sat_f16(A q + B)), the
// arithmetic of the reference's `pro4h` (src/knee/dense8s_kernels.cu:122-139): q is placed exactly
// in an fp16 (1024 + (q + 128) - 1152), one fp16 fma with saturation gives v, and a second fp16
// fma v * 255 + 1024 rounds 255 v to the nearest integer (ties to even) in the low byte.
// a01 / b01: (A, B) of channels c, c+1 as half2; a23 / b23 of c+2, c+3.
DN8_DEV __half2 h2_of(uint32_t x) {
    __half2 h;
    memcpy(&h, &x, 4);
    return h;
}
DN8_DEV uint32_t u32_of(__half2 h) {
    uint32_t x;
    memcpy(&x, &h, 4);
    return x;
}
// The store bytes in offset binary (each byte q + 128, the tile-major store's form).
DN8_DEV uint32_t prologue_f16x4_ob(uint32_t w, uint32_t a01, uint32_t b01, uint32_t a23, uint32_t b23) {
    __half2 lo = h2_of(__byte_perm(w, 0x64646464u, 0x4140));   // fp16 pair 1024 + (q + 128)
    __half2 hi = h2_of(__byte_perm(w, 0x64646464u, 0x4342));
    const __half2 m1152 = h2_of(0xE480E480u), k255 = h2_of(0x5BF85BF8u), k1024 = h2_of(0x64006400u);
    lo = __hadd2(lo, m1152);                             // - 1152: exact q
    hi = __hadd2(hi, m1152);
    lo = __hfma2_sat(lo, h2_of(a01), h2_of(b01));
    hi = __hfma2_sat(hi, h2_of(a23), h2_of(b23));
    lo = __hfma2(lo, k255, k1024);                       // * 255 + 1024
    hi = __hfma2(hi, k255, k1024);
    return __byte_perm(u32_of(lo), u32_of(hi), 0x6420);
}
// The store bytes as signed q (group-major planes, the reference's layout).
DN8_DEV uint32_t prologue_f16x4(uint32_t q4, uint32_t a01, uint32_t b01, uint32_t a23, uint32_t b23) {
    return prologue_f16x4_ob(q4 ^ 0x80808080u, a01, b01, a23, b23);   // signed q -> q + 128
}

// fp32 prologue of one store byte given as w = q + 128 (the reference's `pro16`, :99-120):
// v = sat(fmaf(a, q, b)), u = rint(255 v) as the low byte of fmaf(v, 255, 2^23).
DN8_DEV uint32_t prologue_f32(uint32_t w, float a, float b) {
    const float f = __uint_as_float(0x4B000000u | w) - 8388736.0f;   // exact q
    const float v = __saturatef(fmaf(a, f, b));
    return __float_as_uint(fmaf(v, 255.0f, 8388608.0f)) & 0xFFu;
}
// 4 store bytes in offset binary (q + 128 each)
DN8_DEV uint32_t prologue_f32x4_ob(uint32_t w4, const float2* ab) {
    uint32_t r = 0;
#pragma unroll
    for (int k = 0; k < 4; ++k) r |= prologue_f32((w4 >> (8 * k)) & 0xFFu, ab[k].x, ab[k].y) << (8 * k);
    return r;
}
// 4 store bytes as signed q
DN8_DEV uint32_t prologue_f32x4(uint32_t q4, const float2* ab) { return prologue_f32x4_ob(q4 ^ 0x80808080u, ab); }

// Two fp16 pixels (one half2 word) -> two u8 in the low 16 bits: rint(255 sat(x)) computed in fp32
// (the reference's `u8pair`, dense8s_kernels.cu:3631-3639).
DN8_DEV uint32_t u8_of_f16x2(uint32_t h2) {
    const float a = __half2float(__ushort_as_half(static_cast<unsigned short>(h2 & 0xFFFFu)));
    const float b = __half2float(__ushort_as_half(static_cast<unsigned short>(h2 >> 16)));
    const uint32_t qa = __float_as_uint(fmaf(__saturatef(a), 255.0f, 12582912.0f));
    const uint32_t qb = __float_as_uint(fmaf(__saturatef(b), 255.0f, 12582912.0f));
    return __byte_perm(qa, qb, 0x0040) & 0xFFFFu;
}

}  // namespace dn8
