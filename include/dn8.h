/* dn8.h -- C ABI of libdn8b200.so, the Blackwell (sm_100a) INT8 DenseNet169 encoder.
 *
 * Two levels, both plain C (pointers, sizes, integer status; no exceptions cross the ABI):
 *
 * 1. Kernel level. The reference binds each INT8 kernel by name through its ctypes driver-API
 *    wrapper `cudart.Function.launch(grid, block, [struct], stream, shared)`
 *    (src/knee/cudart.py:138-153) with a by-value argument struct (`KArg`
 *    src/knee/dense8s_kernels.cu:147-158, `C2Arg` :1936-1942). Here each kernel family is one
 *    host function taking an argument struct of the same meaning plus the caller's stream; the
 *    library picks grid, block and shared memory itself. All pointers are DEVICE pointers. The
 *    weight / scale tables are the reference pack tables (`kernel_params`,
 *    src/knee/dense8s.py:457-519) unchanged.
 *
 * 2. Engine level. Replaces `Dense8SEncoder` (src/knee/dense8s.py:944-1488): one handle per
 *    (GPU, seed) owns the device copies of the pack tables and the block arenas; `dn8_forward`
 *    enqueues one whole pass (stem, 82 dense layers, 3 transitions, pooling + head) on the
 *    caller's stream without host synchronisation or allocation, so it can be captured in a CUDA
 *    graph. A handle is not thread-safe; distinct handles are independent.
 *
 * Block stores. Activations (int8 q, 32-channel groups) are either the reference's group-major
 * planes [G][N*HW][32] of signed bytes, or (tile_groups > 0 in the argument structs) a tile-major
 * block store [ceil(N*HW/128)][tile_groups][128][32]: 128 consecutive pixels per tile, all of a
 * tile's groups contiguous, each byte q + 128 (offset binary: the prologue's own input form, so
 * its readers skip the sign flip of every byte). The engine keeps every block in that form;
 * dn8_engine_store returns signed q.
 *
 * Status codes: DN8_OK, DN8_EINVAL (bad argument or unsupported geometry; the reference raises
 * ValueError), DN8_ECUDA (CUDA runtime error; reference `cudart.CudaError`), DN8_EDEVICE (a kernel
 * reported an error through its error word: a bounded device-side wait gave up). The last error
 * message of a handle (or of the calling thread, for the kernel level) is dn8_last_error().
 */
#ifndef DN8_H
#define DN8_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define DN8_OK 0
#define DN8_EINVAL 1
#define DN8_ECUDA 2
#define DN8_EDEVICE 3

typedef void* dn8_stream; /* a cudaStream_t; NULL = legacy default stream */

/* ---- kernel level -------------------------------------------------------------------------- */

/* conv1 of dense layer (b, l): replaces `conv1_w64_pl(KArg)` / `conv1_u*(KArg)` (reference
 * src/knee/dense8s_kernels.cu:479-627, launched by `Dense8SEncoder._c1_item` src/knee/dense8s.py:1205-1240).
 * u = prologue(q) per channel, acc = sum_c W[o,c] u_c (int32), out = rint(255 sat(g_o acc + d_o)).
 * Store: in0 [G0][N][HW][32] int8 (group-major: unlike the reference's [N][G0][HW][32], every
 * 32-channel group of a 128-pixel tile is one contiguous 4 KB run), seg [L][N][HW][32] int8
 * (groups G0.. read from seg).
 * Output: the u8 bottleneck as 8 planes of 16 channels, [8][N*HW][16].
 * G <= 70 (2240 input channels): the weights stay resident in shared memory, on single CTAs up to
 * G = 37 and on clusters of two CTAs (half the weights each) above. */
typedef struct dn8_conv1_args {
    const int8_t* in0;
    const int8_t* seg;
    const int8_t* w;    /* L*_w1 [G][128][32] after dn8_prepare_conv1_weights (G * 4096 bytes) */
    const void* ab;     /* prologue table: L*_abh [G*16][4] fp16 (prologue_f16 = 1) or L*_ab [G*32][2] float */
    const float* gd;    /* L*_gdu: [128][2] float */
    uint8_t* out;       /* [8][N*HW][16] */
    int32_t* err;       /* device error word (0 = none) or NULL */
    int32_t G0, G, N, HW;
    int32_t prologue_f16;
    /* 0: in0 / seg are the reference's group-major planes [G0][N*HW][32] / [G-G0][N*HW][32].
     * > 0: in0 is a tile-major block store [ceil(N*HW/128)][tile_groups][128][32] (128 consecutive
     * pixels per tile, all of a tile's groups contiguous, bytes q + 128) holding groups 0 .. G-1; seg
     * and G0 are unused. */
    int32_t tile_groups;
} dn8_conv1_args;
int dn8_conv1(const dn8_conv1_args* a, dn8_stream stream);

/* conv2 of dense layer (b, l): replaces `conv2_t8x32_pl` / `conv2_t16x16_pl(C2Arg)` (reference
 * :2679-2832, `_c2_item` src/knee/dense8s.py:1274-1290). 3x3 pad-1 conv 128 -> 32 on the u8
 * bottleneck, q = rint(clamp(acc * sc_o, +-127)) written into the store slot [N][HW][32] or, with
 * tile_groups > 0, into group `group` of a tile-major block store. Requires W <= 128. */
typedef struct dn8_conv2_args {
    const uint8_t* x;   /* bottleneck planes [8][N*H*W][16] */
    const int8_t* w;    /* L*_w2k [4][9][32][32] after dn8_prepare_conv2_weights (36864 bytes) */
    const float* sc;    /* L*_c2u: [32] float */
    int8_t* out;        /* store slot [N][H*W][32], or the tile-major block store */
    int32_t* err;
    int32_t N, H, W;
    /* 0: out is the slot. > 0: out is a tile-major block store [ceil(N*H*W/128)][tile_groups][128][32]
     * (128 consecutive pixels per tile, all of a tile's groups contiguous, bytes q + 128) and this
     * layer writes its group `group` (< tile_groups). */
    int32_t tile_groups, group;
} dn8_conv2_args;
int dn8_conv2(const dn8_conv2_args* a, dn8_stream stream);

/* transition of block b: replaces `trans_w0` / `trans_w1(KArg)` (reference :3077-3268) and the
 * integer form `trans_q128(KArg)` (:176-422, MODE 1), launched by `_trans_item`
 * (src/knee/dense8s.py:1242-1272). Prologue as conv1 on all G = c_tot / 32 groups, 1x1 conv
 * c_tot -> c_tot / 2, the four accumulators of every 2x2 square summed exactly (int32), then
 * q = rint(clamp(k_o * s, +-127)), k = T*_gd[o][0], into the next block's group-major in0
 * [c_tot/64][N][H*W/4][32]. c_tot a multiple of 256 (G % 8 == 0), H and W even. */
typedef struct dn8_trans_args {
    const int8_t* in0;
    const int8_t* seg;
    const int8_t* w;    /* T*_w [G][c_out][32] after dn8_prepare_trans_weights (G * c_out * 32 bytes) */
    const void* ab;     /* T*_abh (prologue_f16 = 1) or T*_ab */
    const float* gd;    /* T*_gd: [c_out][2] float */
    int8_t* out;        /* next block's in0 */
    int32_t* err;
    int32_t G0, G, N, H, W;
    int32_t prologue_f16;
    /* > 0: in0 is a tile-major block store [ceil(N*H*W/128)][tile_groups][128][32] (bytes q + 128)
     * holding groups 0 .. G-1 (seg and G0 unused). */
    int32_t tile_groups;
    /* > 0: out is the next block's tile-major store [ceil(N*H*W/4/128)][out_tile_groups][128][32]
     * (bytes q + 128); the transition writes its groups 0 .. c_out/32 - 1. */
    int32_t out_tile_groups;
} dn8_trans_args;
int dn8_trans(const dn8_trans_args* a, dn8_stream stream);

/* stem: replaces the reference's TensorRT fp16 stem + `quant_seg` and its exact INT8 form
 * `stem_i8` (src/knee/dense8s_kernels.cu:3641-3771, formula `stem_q_i8` src/knee/dense8s.py:625-643),
 * fused with the input producer `gather_u8_to_f16` (src/knee/data/fused_uint8.py:480-505).
 * Pixels: x_u8 = 0: fp16 windows [N][3][H][W], u = rint(255 sat(x)); x_u8 = 1: uint8 planes
 * [P][H][W] gathered through src[N][4] = {plane of channel 0, 1, 2, unused}, u = the byte.
 * flags[n] bit 0 (optional array): horizontal flip of image n. 7x7/2 pad-3 conv with the int8
 * weights, q = rint(clamp(fmaf(acc, k_o, c_o), 0, 127)) (S_kc = [k(64), c(64)]), 3x3/2 pad-1
 * max-pool, into block 1's group-major input [2][N][H/4 * W/4][32]. H, W multiples of 4, W <= 512. */
typedef struct dn8_stem_args {
    const void* x;
    const int32_t* src;    /* x_u8 = 1: [N][4] plane indices */
    const int32_t* flags;  /* [N] or NULL */
    const int8_t* w;       /* S_w8 [64][176] after dn8_prepare_stem_weights (14336 bytes) */
    const float* kc;       /* S_kc [128] */
    int8_t* out;
    int32_t* err;
    int32_t N, H, W;
    int32_t x_u8;
    int32_t n_alloc;       /* images the output groups are laid out for (>= N; 0 = N) */
    /* > 0: out is block 1's tile-major store [ceil(n_alloc*H*W/16/128)][tile_groups][128][32]
     * (bytes q + 128); the stem writes its groups 0 and 1. */
    int32_t tile_groups;
} dn8_stem_args;
int dn8_stem(const dn8_stem_args* a, dn8_stream stream);

/* global pooling + linear head: replaces `final_q` (reference :2304-2323, launched at
 * src/knee/dense8s.py:1379-1385) and adds the benchmark head (linear C -> n_out, mean over the
 * slices of a view). features = mean over pixels of relu(a_c q + b_c) (F_ab, the reference's
 * summation order); logits = features . Hw^T + Hb (fp32); view_logits[v] = mean of the logits of
 * images v*per_view .. v*per_view + per_view - 1. A cluster of four CTAs per image; G <= 72
 * (2304 channels), n_out <= 64. */
typedef struct dn8_head_args {
    const int8_t* in0;      /* last block's input groups, group-major [G0][N][HW][32] */
    const int8_t* seg;      /* its layer segments [L][N][HW][32] */
    const float* fab;       /* F_ab [C][2] */
    float* feat;            /* [N][C] float, or NULL */
    const float* hw;        /* [n_out][C] float, or NULL (no head) */
    const float* hb;        /* [n_out] */
    float* logits;          /* [N][n_out] */
    float* view_logits;     /* [N / per_view][n_out], or NULL (needs hw: rejected without a head) */
    int32_t* tickets;       /* [N / per_view] zero-initialised device counters (left zeroed) */
    int32_t G0, G, N, HW, n_out, per_view;
    int32_t n_alloc;        /* images the store groups are laid out for (>= N; 0 = N) */
    /* > 0: in0 is the last block's tile-major store [ceil(n_alloc*HW/128)][tile_groups][128][32]
     * (bytes q + 128) holding groups 0 .. G-1 (seg and G0 unused). */
    int32_t tile_groups;
} dn8_head_args;
int dn8_head(const dn8_head_args* a, dn8_stream stream);

/* dn8_head without a caller-provided ticket array (no counterpart in the reference): the per-view
 * counters live in a scratch array built into the library, DN8_HEAD_SCRATCH_VIEWS int32 per device,
 * so the call allocates nothing. a->tickets must be NULL; N / per_view above DN8_HEAD_SCRATCH_VIEWS
 * is rejected with DN8_EINVAL before any CUDA call. The scratch starts at zero and every completed
 * call leaves it zero. The first call on a device looks the scratch up (cudaGetSymbolAddress, which
 * can load the module on that device): make it before any stream capture. Calls that may overlap
 * (on several streams, or several threads, of one device) share the scratch and race: issue them
 * in order on one stream. */
#define DN8_HEAD_SCRATCH_VIEWS 4096
int dn8_head_noalloc(const dn8_head_args* a, dn8_stream stream);

/* geometric test-time view: replaces `affine_windows` (src/knee/tta.py:131-149; zoom `scale` about
 * the centre, shift (tx, ty) as fractions of the side, bilinear, zero outside, align_corners =
 * False, in fp16) applied to the windows the reference gathers from the uint8 volume
 * (`gather_u8_to_f16`, src/knee/data/fused_uint8.py:480-505). Reads the uint8 planes [P][H][W]
 * through src[N][4] (planes of channels 0-2), flags[N] bit 0 = mirror the window first; writes the
 * fp16 windows [N][3][H][W] that dn8_stem (x_u8 = 0) or the engine read. W a multiple of 16,
 * scale >= 0.25. */
typedef struct dn8_zoom_args {
    const uint8_t* planes;
    const int32_t* src;
    const int32_t* flags;   /* [N] or NULL */
    uint16_t* out;          /* fp16 [N][3][H][W] */
    int32_t* err;
    int32_t N, H, W;
    double scale, tx, ty;   /* as the reference's Python floats */
} dn8_zoom_args;
int dn8_zoom(const dn8_zoom_args* a, dn8_stream stream);

/* ---- weight preparation (host memory to host memory, once per pack) ------------------------
 * The kernels read their weights with bulk copies straight into the tensor cores' shared-memory
 * operand layout; these functions permute the reference pack tables into that layout. */
int dn8_prepare_conv1_weights(const int8_t* w1, int32_t G, uint8_t* out);               /* G*4096 B */
int dn8_prepare_trans_weights(const int8_t* tw, int32_t G, int32_t cout, uint8_t* out); /* G*cout*32 B */
int dn8_prepare_conv2_weights(const int8_t* w2k, uint8_t* out);                         /* 36864 B */
int dn8_prepare_stem_weights(const int8_t* w8, uint8_t* out);                           /* 14336 B */

/* ---- engine level ------------------------------------------------------------------------- */

typedef struct dn8_table {  /* one pack table, by the reference's name (`kernel_params`) */
    const char* name;       /* e.g. "L0_3_w1", "T1_abh", "F_ab", "S_w8", "S_kc", "H_w" */
    const void* data;       /* host memory, the reference's layout and dtype */
    int64_t nbytes;
} dn8_table;

typedef struct dn8_pack_desc {  /* the pack `meta` (src/knee/dense8s.py:810-831) as plain fields */
    int32_t n;              /* images per pass (meta "n") */
    int32_t img, in_ch, n_blocks;
    int32_t c0[4], h[4], w[4], L[4], trans[4];
    int32_t trans_f16[4];   /* transition prologue: 1 = T*_abh (fp16), 0 = T*_ab (fp32) */
    const int8_t* c1_f16[4];/* per dense layer: 1 = L*_abh (fp16 prologue), 0 = L*_ab */
    int32_t n_out;          /* head outputs (tables H_w, H_b); 0 = features only */
    const dn8_table* tables;
    int32_t n_tables;
} dn8_pack_desc;

typedef struct dn8_engine dn8_engine;

typedef struct dn8_input {  /* the pixels of one forward call */
    const void* x;          /* x_u8 = 0: fp16 [n][3][img][img]; x_u8 = 1: uint8 planes [P][img][img] */
    const int32_t* src;     /* x_u8 = 1: device [n][4] plane indices of the 3 channels (+ unused) */
    const int32_t* flags;   /* device [n] (bit 0: horizontal flip) or NULL */
    int32_t x_u8;
} dn8_input;

/* Validates and uploads the pack; allocates arenas for `n` images per pass on `device`. */
int dn8_engine_create(const dn8_pack_desc* pack, int device, dn8_engine** out);
void dn8_engine_destroy(dn8_engine* e);
/* Enqueues ceil(n / pass) passes on `stream`: features [n][C] (float, NULL to skip), logits
 * [n][n_out] and view_logits [n / per_view][n_out] (NULL to skip). All pointers are device
 * pointers. No allocation and no host synchronisation: capturable in a CUDA graph. */
int dn8_engine_forward(dn8_engine* e, const dn8_input* in, int32_t n, float* feat, float* logits,
                       float* view_logits, int32_t per_view, dn8_stream stream);
/* Synchronises `stream`, then reads (and clears) the device error word: DN8_EDEVICE if a kernel gave
 * up a bounded wait since the last check. */
int dn8_engine_check(dn8_engine* e, dn8_stream stream);
/* Enqueues one pass of n (<= pass size) images that stops after the dense layers of block
 * `last_block` (its transition and, for the last block, the pooling + head are not run), so that
 * dn8_engine_store reads blocks last_block - 1 and last_block as the pass left them. The reference's
 * `Dense8SEncoder.trace` (src/knee/dense8s.py:1509-1546) copies the store after every block; passes
 * are deterministic, so a partial pass and a full one give every block's store. */
int dn8_engine_forward_to(dn8_engine* e, const dn8_input* in, int32_t n, int32_t last_block, dn8_stream stream);
/* Launches one kernel of a pass -- kind DN8_K_CONV1 or DN8_K_CONV2 of dense layer `layer` of block
 * `block`, or DN8_K_TRANS of block `block` -- on the engine's arenas exactly as a pass does, without
 * programmatic dependence on the previous launch. For timing (the reference's `time_layers` times
 * its stored launch items, src/knee/dense8s.py:1583-1596): it reads whatever the last pass left
 * and overwrites what that kernel writes. No allocation, no synchronisation. */
int dn8_engine_launch(dn8_engine* e, int32_t kind, int32_t block, int32_t layer, dn8_stream stream);
/* Copies store segment j of block b (j = 0: the block input groups [G0][n][HW][32]; j >= 1: the
 * output of dense layer j-1, [n][HW][32]) to dst (device or host memory) as signed q, enqueued on
 * `stream` (a host dst holds the bytes once the stream has reached this point). Valid for the last
 * two blocks of the last pass (blocks alternate between two arenas). */
int dn8_engine_store(const dn8_engine* e, int32_t block, int32_t j, int8_t* dst, dn8_stream stream);
/* One pass of n (<= pass size) images with a CUDA event after every launch (the reference's
 * `Dense8SEncoder.profile`, src/knee/dense8s.py:1548-1563): out[k] = kind, block, layer and device
 * milliseconds of launch k, *n_launches = launches of the pass. Synchronises `stream`. */
#define DN8_K_STEM 0
#define DN8_K_CONV1 1
#define DN8_K_CONV2 2
#define DN8_K_TRANS 3
#define DN8_K_HEAD 4
typedef struct dn8_launch_info {
    int32_t kind, block, layer;
    float ms;
} dn8_launch_info;
int dn8_engine_profile(dn8_engine* e, const dn8_input* in, int32_t n, float* feat, dn8_launch_info* out,
                       int32_t max_out, int32_t* n_launches, dn8_stream stream);
const char* dn8_engine_error(const dn8_engine* e);
int64_t dn8_engine_device_bytes(const dn8_engine* e);

/* ---- test hook (failure detection without a GPU fault) -------------------------------------
 * Arms the next dn8_conv1 launch of the process (kernel level or inside an engine pass) with a short
 * wait limit (`wait_limit_cycles` SM cycles instead of ~2^32) and, for fault = 1, makes the store
 * producer of its first CTA (or CTA pair) announce raw stage 0 of its first tile but never copy it.
 * That CTA's consumers then give up their bounded wait: the launch sets its error word (a dn8_conv1
 * `err` array, or the engine's: dn8_engine_check returns DN8_EDEVICE), every role leaves its loop,
 * the kernel frees its tensor memory and returns, and the context stays usable. fault = 0 disarms.
 * No counterpart in the reference; never armed outside tests. */
int dn8_test_inject_wait_fault(int32_t fault, int64_t wait_limit_cycles);

const char* dn8_last_error(void);   /* message of the calling thread's last failed call */
int dn8_device_sms(int device);     /* SM count used to size persistent grids (0 on error) */

#ifdef __cplusplus
}
#endif
#endif /* DN8_H */
