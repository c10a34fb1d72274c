// engine.cu -- the encoder runner behind the C ABI: the native replacement of the reference's
// `Dense8SEncoder` (src/knee/dense8s.py:944-1488). One engine per (GPU, pack):
//   * the pack tables (reference names and layouts) are validated, permuted into the kernels'
//     operand layouts once, and copied to the device in one allocation;
//   * two alternating block arenas as in the reference (`_buffers`, dense8s.py:1073-1092): block b
//     lives in arena b % 2 and its transition writes the next block's input into the other one.
//     Every block store is tile-major [ceil(n_cap HW / 128)][Gt][128][32] (Gt = G0 + L groups: the
//     block input groups first, then one group per dense layer; all groups of 128 consecutive pixels
//     contiguous), so segment l of block b is group G0 + l of every tile and each conv1 stage reads
//     one contiguous run;
//   * a pass always runs the full capacity n_cap through the dense blocks (fixed shapes: a pass is
//     capturable in a CUDA graph and its tensor maps stay valid); only the stem and the head see
//     the real image count, so short batches cost one pass like the reference's padded blocks;
//   * dn8_engine_forward only enqueues kernels on the caller's stream: no allocation, no host sync.
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <string>
#include <unordered_map>
#include <vector>

#include <new>

#include "dn8_kernels.h"

struct dn8_engine {
    int device = 0, sms = 0, n = 0, img = 0, n_blocks = 0, n_out = 0;
    int c0[4], h[4], w[4], L[4], trans[4], trans_f16[4];
    std::vector<int8_t> c1_f16[4];
    uint8_t* tables = nullptr;          // device: every prepared table
    int8_t* arena[2] = {nullptr, nullptr};
    uint8_t* bott = nullptr;            // conv1 -> conv2 bottleneck planes [8][n * HW][16]
    int32_t* err = nullptr;             // device error word
    int32_t* tickets = nullptr;         // head per-view counters
    size_t dev_bytes = 0;
    struct Layer { const uint8_t* w1; const void* ab; const float* gd; const uint8_t* w2; const float* c2; };
    std::vector<Layer> layers[4];
    const uint8_t* tw[4]; const void* tab[4]; const float* tgd[4];
    const float* fab = nullptr; const uint8_t* sw = nullptr; const float* kc = nullptr;
    const float* hw = nullptr; const float* hb = nullptr;
    dn8::Conv2Plan c2plan[4];
    std::string error;
    // profiling: an event after every launch of one pass, with (kind, block, layer) of the launch
    std::vector<cudaEvent_t> events;
    std::vector<dn8_launch_info> rec;
    bool profiling = false;
};

namespace {

int efail(dn8_engine* e, int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    if (e) e->error = buf;
    return code;
}

struct HostTables {
    std::unordered_map<std::string, const dn8_table*> by_name;
    const dn8_table* get(const std::string& name) const {
        auto it = by_name.find(name);
        return it == by_name.end() ? nullptr : it->second;
    }
};

size_t align256(size_t x) { return (x + 255) / 256 * 256; }

}  // namespace

extern "C" {

const char* dn8_engine_error(const dn8_engine* e) { return e ? e->error.c_str() : "null engine"; }
int64_t dn8_engine_device_bytes(const dn8_engine* e) { return e ? static_cast<int64_t>(e->dev_bytes) : 0; }

void dn8_engine_destroy(dn8_engine* e) {
    if (e == nullptr) return;
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(e->device);
    for (cudaEvent_t ev : e->events) cudaEventDestroy(ev);
    cudaFree(e->tables);
    cudaFree(e->arena[0]);
    cudaFree(e->arena[1]);
    cudaFree(e->bott);
    cudaFree(e->err);
    cudaFree(e->tickets);
    cudaSetDevice(prev);
    delete e;
}

}  // extern "C"

static int engine_create(const dn8_pack_desc* p, int device, dn8_engine** out) {
    if (out == nullptr || p == nullptr) return DN8_EINVAL;
    *out = nullptr;
    dn8_engine* e = new dn8_engine();
    e->device = device;
    auto bail = [&](int code) {
        if (code != DN8_OK) {
            std::string msg = e->error;
            dn8_engine_destroy(e);
            // keep the message reachable through the thread-local channel of the kernel level
            dn8::set_last_error(msg.c_str());
        }
        return code;
    };
    if (p->n < 1 || p->n_blocks < 1 || p->n_blocks > 4 || p->in_ch != 3 || p->img < 16 || p->img % 32)
        return bail(efail(e, DN8_EINVAL, "pack geometry: n=%d blocks=%d in_ch=%d img=%d", p->n, p->n_blocks,
                          p->in_ch, p->img));
    e->n = p->n; e->img = p->img; e->n_blocks = p->n_blocks; e->n_out = p->n_out;
    for (int b = 0; b < p->n_blocks; ++b) {
        e->c0[b] = p->c0[b]; e->h[b] = p->h[b]; e->w[b] = p->w[b]; e->L[b] = p->L[b];
        e->trans[b] = p->trans[b]; e->trans_f16[b] = p->trans_f16[b];
        if (p->c0[b] % 32 || p->L[b] < 1 || p->h[b] < 1 || p->w[b] < 1 || p->w[b] > 128 ||
            (p->trans[b] && ((p->c0[b] + 32 * p->L[b]) % 256 || p->h[b] % 2 || p->w[b] % 2)))
            return bail(efail(e, DN8_EINVAL, "block %d geometry c0=%d L=%d h=%d w=%d not supported", b, p->c0[b],
                              p->L[b], p->h[b], p->w[b]));
        e->c1_f16[b].assign(p->c1_f16[b], p->c1_f16[b] + p->L[b]);
    }
    if (p->h[0] * 4 != p->img || p->w[0] * 4 != p->img || p->c0[0] != 64)
        return bail(efail(e, DN8_EINVAL, "block 0 must be img/4 x img/4 with 64 input channels"));
    for (int b = 0; b < p->n_blocks; ++b) {
        // every block but the last ends in a transition that halves the map and the channels
        const bool last = b == p->n_blocks - 1;
        if (p->trans[b] != (last ? 0 : 1) ||
            (!last && (p->c0[b + 1] * 2 != p->c0[b] + 32 * p->L[b] || p->h[b + 1] * 2 != p->h[b] ||
                       p->w[b + 1] * 2 != p->w[b])))
            return bail(efail(e, DN8_EINVAL, "block %d: transitions must chain the blocks (c0 = c_tot / 2, "
                              "half the side) and the last block has none", b));
    }
    HostTables ht;
    for (int i = 0; i < p->n_tables; ++i) ht.by_name[p->tables[i].name] = &p->tables[i];

    // ---- host staging of every prepared table, then one device copy ----
    std::vector<uint8_t> stage;
    auto reserve = [&](size_t bytes) {
        const size_t off = align256(stage.size());
        stage.resize(off + bytes);
        return off;
    };
    std::string bad;
    auto need = [&](const std::string& name, size_t bytes) -> const dn8_table* {
        const dn8_table* t = ht.get(name);
        if (t == nullptr || t->data == nullptr || static_cast<size_t>(t->nbytes) != bytes) {
            if (bad.empty())
                bad = name + (t == nullptr ? " missing" : " has " + std::to_string(t->nbytes) + " bytes, expected " +
                                                               std::to_string(bytes));
            return nullptr;
        }
        return t;
    };
    auto copy_raw = [&](const dn8_table* t) {
        const size_t off = reserve(static_cast<size_t>(t->nbytes));
        std::memcpy(stage.data() + off, t->data, static_cast<size_t>(t->nbytes));
        return off;
    };
    struct LOff { size_t w1, ab, gd, w2, c2; };
    std::vector<LOff> loff[4];
    size_t toff[4][3];
    for (int b = 0; b < e->n_blocks; ++b) {
        for (int l = 0; l < e->L[b]; ++l) {
            const int cin = e->c0[b] + 32 * l, G = cin / 32;
            const std::string k = "L" + std::to_string(b) + "_" + std::to_string(l) + "_";
            const bool f16 = e->c1_f16[b][l] != 0;
            const dn8_table* w1 = need(k + "w1", static_cast<size_t>(G) * 4096);
            const dn8_table* ab = f16 ? need(k + "abh", static_cast<size_t>(cin) * 4) : need(k + "ab", static_cast<size_t>(cin) * 8);
            const dn8_table* gd = need(k + "gdu", 128 * 8);
            const dn8_table* w2 = need(k + "w2k", 36864);
            const dn8_table* c2 = need(k + "c2u", 32 * 4);
            if (!bad.empty()) return bail(efail(e, DN8_EINVAL, "pack table %s", bad.c_str()));
            LOff o;
            o.w1 = reserve(static_cast<size_t>(G) * 4096);
            dn8_prepare_conv1_weights(static_cast<const int8_t*>(w1->data), G, stage.data() + o.w1);
            o.ab = copy_raw(ab);
            o.gd = copy_raw(gd);
            o.w2 = reserve(36864);
            dn8_prepare_conv2_weights(static_cast<const int8_t*>(w2->data), stage.data() + o.w2);
            o.c2 = copy_raw(c2);
            loff[b].push_back(o);
        }
        if (e->trans[b]) {
            const int ctot = e->c0[b] + 32 * e->L[b], G = ctot / 32, cout = ctot / 2;
            const std::string k = "T" + std::to_string(b) + "_";
            const dn8_table* tw = need(k + "w", static_cast<size_t>(G) * cout * 32);
            const dn8_table* ab = e->trans_f16[b] ? need(k + "abh", static_cast<size_t>(ctot) * 4)
                                                  : need(k + "ab", static_cast<size_t>(ctot) * 8);
            const dn8_table* gd = need(k + "gd", static_cast<size_t>(cout) * 8);
            if (!bad.empty()) return bail(efail(e, DN8_EINVAL, "pack table %s", bad.c_str()));
            toff[b][0] = reserve(static_cast<size_t>(G) * cout * 32);
            dn8_prepare_trans_weights(static_cast<const int8_t*>(tw->data), G, cout, stage.data() + toff[b][0]);
            toff[b][1] = copy_raw(ab);
            toff[b][2] = copy_raw(gd);
        }
    }
    const int last = e->n_blocks - 1;
    const int C = e->c0[last] + 32 * e->L[last];
    const dn8_table* fab = need("F_ab", static_cast<size_t>(C) * 8);
    const dn8_table* sw8 = need("S_w8", 64 * 176);
    const dn8_table* skc = need("S_kc", 128 * 4);
    const dn8_table* hw = e->n_out > 0 ? need("H_w", static_cast<size_t>(e->n_out) * C * 4) : nullptr;
    const dn8_table* hb = e->n_out > 0 ? need("H_b", static_cast<size_t>(e->n_out) * 4) : nullptr;
    if (!bad.empty()) return bail(efail(e, DN8_EINVAL, "pack table %s", bad.c_str()));
    const size_t o_fab = copy_raw(fab);
    const size_t o_sw = reserve(14336);
    dn8_prepare_stem_weights(static_cast<const int8_t*>(sw8->data), stage.data() + o_sw);
    const size_t o_kc = copy_raw(skc);
    const size_t o_hw = hw ? copy_raw(hw) : 0, o_hb = hb ? copy_raw(hb) : 0;

    // ---- device memory ----
    int prev = 0;
    cudaGetDevice(&prev);
    cudaError_t ce = cudaSetDevice(device);
    if (ce != cudaSuccess) return bail(efail(e, DN8_ECUDA, "cudaSetDevice(%d): %s", device, cudaGetErrorString(ce)));
    auto dev_alloc = [&](void** ptr, size_t bytes) {
        ce = cudaMalloc(ptr, bytes > 0 ? bytes : 16);
        if (ce == cudaSuccess) e->dev_bytes += bytes;
        return ce == cudaSuccess;
    };
    size_t arena_bytes[2] = {0, 0}, hw_max = 0;
    for (int b = 0; b < e->n_blocks; ++b) {
        const size_t hwb = static_cast<size_t>(e->h[b]) * e->w[b];
        const size_t groups = e->c0[b] / 32 + e->L[b];
        const size_t tiles = (static_cast<size_t>(e->n) * hwb + 127) / 128;
        arena_bytes[b % 2] = std::max(arena_bytes[b % 2], tiles * groups * 4096);
        hw_max = std::max(hw_max, hwb);
    }
    bool ok = dev_alloc(reinterpret_cast<void**>(&e->tables), stage.size()) &&
              dev_alloc(reinterpret_cast<void**>(&e->arena[0]), arena_bytes[0]) &&
              dev_alloc(reinterpret_cast<void**>(&e->arena[1]), arena_bytes[1]) &&
              dev_alloc(reinterpret_cast<void**>(&e->bott), static_cast<size_t>(e->n) * hw_max * 128) &&
              dev_alloc(reinterpret_cast<void**>(&e->err), 256) &&
              dev_alloc(reinterpret_cast<void**>(&e->tickets), static_cast<size_t>(e->n) * 4);
    if (!ok) {
        cudaSetDevice(prev);
        return bail(efail(e, DN8_ECUDA, "device allocation (%zu bytes so far): %s", e->dev_bytes, cudaGetErrorString(ce)));
    }
    ce = cudaMemcpy(e->tables, stage.data(), stage.size(), cudaMemcpyHostToDevice);
    if (ce == cudaSuccess) ce = cudaMemset(e->err, 0, 256);
    if (ce == cudaSuccess) ce = cudaMemset(e->tickets, 0, static_cast<size_t>(e->n) * 4);
    // zero the arenas once: a short pass leaves the padded images' inputs as they are, and they
    // must hold defined bytes
    if (ce == cudaSuccess) ce = cudaMemset(e->arena[0], 0, arena_bytes[0] ? arena_bytes[0] : 16);
    if (ce == cudaSuccess) ce = cudaMemset(e->arena[1], 0, arena_bytes[1] ? arena_bytes[1] : 16);
    if (ce != cudaSuccess) {
        cudaSetDevice(prev);
        return bail(efail(e, DN8_ECUDA, "table upload: %s", cudaGetErrorString(ce)));
    }
    auto T = [&](size_t off) { return e->tables + off; };
    for (int b = 0; b < e->n_blocks; ++b) {
        for (const LOff& o : loff[b])
            e->layers[b].push_back({T(o.w1), T(o.ab), reinterpret_cast<const float*>(T(o.gd)), T(o.w2),
                                    reinterpret_cast<const float*>(T(o.c2))});
        if (e->trans[b]) {
            e->tw[b] = T(toff[b][0]);
            e->tab[b] = T(toff[b][1]);
            e->tgd[b] = reinterpret_cast<const float*>(T(toff[b][2]));
        }
        dn8_conv2_args a2{};
        a2.x = e->bott; a2.N = e->n; a2.H = e->h[b]; a2.W = e->w[b];
        ce = dn8::prepare_conv2(&e->c2plan[b], a2);
        if (ce != cudaSuccess) {
            cudaSetDevice(prev);
            return bail(efail(e, DN8_ECUDA, "conv2 tensor map of block %d: %s", b, cudaGetErrorString(ce)));
        }
    }
    e->fab = reinterpret_cast<const float*>(T(o_fab));
    e->sw = T(o_sw);
    e->kc = reinterpret_cast<const float*>(T(o_kc));
    if (hw) {
        e->hw = reinterpret_cast<const float*>(T(o_hw));
        e->hb = reinterpret_cast<const float*>(T(o_hb));
    }
    cudaDeviceGetAttribute(&e->sms, cudaDevAttrMultiProcessorCount, device);
    cudaSetDevice(prev);
    *out = e;
    return DN8_OK;
}

extern "C" {

// host allocation failures (std::bad_alloc) end as a status, not as an exception through the C ABI
int dn8_engine_create(const dn8_pack_desc* p, int device, dn8_engine** out) {
    try {
        return engine_create(p, device, out);
    } catch (const std::exception& ex) {
        dn8::set_last_error(ex.what());
        return DN8_EINVAL;
    }
}

// In profiling mode, records an event after a launch of (kind, block, layer).
static void mark(dn8_engine* e, int kind, int block, int layer, cudaStream_t st) {
    if (!e->profiling) return;
    const size_t i = e->rec.size();
    if (i + 1 >= e->events.size()) return;
    cudaEventRecord(e->events[i + 1], st);
    e->rec.push_back({kind, block, layer, 0.0f});
}

// The dense-layer and transition launches of a pass, on the engine's arenas (pdl: programmatic
// dependent launch on the previous kernel of the pass).
static cudaError_t launch_conv1_of(dn8_engine* e, int b, int l, cudaStream_t st, bool pdl) {
    const int G0 = e->c0[b] / 32;
    const dn8_engine::Layer& ly = e->layers[b][l];
    dn8_conv1_args c1{};
    c1.in0 = e->arena[b % 2]; c1.seg = nullptr; c1.w = reinterpret_cast<const int8_t*>(ly.w1); c1.ab = ly.ab;
    c1.gd = ly.gd; c1.out = e->bott; c1.err = e->err; c1.G0 = G0; c1.G = G0 + l; c1.N = e->n;
    c1.HW = e->h[b] * e->w[b]; c1.prologue_f16 = e->c1_f16[b][l];
    c1.tile_groups = G0 + e->L[b];
    return dn8::launch_conv1(c1, e->sms, st, pdl);
}

static cudaError_t launch_conv2_of(dn8_engine* e, int b, int l, cudaStream_t st, bool pdl) {
    const int G0 = e->c0[b] / 32;
    const dn8_engine::Layer& ly = e->layers[b][l];
    dn8_conv2_args c2{};
    c2.x = e->bott; c2.w = reinterpret_cast<const int8_t*>(ly.w2); c2.sc = ly.c2;
    c2.out = e->arena[b % 2]; c2.err = e->err;
    c2.N = e->n; c2.H = e->h[b]; c2.W = e->w[b];
    c2.tile_groups = G0 + e->L[b]; c2.group = G0 + l;
    return dn8::launch_conv2(e->c2plan[b], c2, e->sms, st, pdl);
}

static cudaError_t launch_trans_of(dn8_engine* e, int b, cudaStream_t st, bool pdl) {
    const int G0 = e->c0[b] / 32, Gt = G0 + e->L[b];
    dn8_trans_args t{};
    t.in0 = e->arena[b % 2]; t.seg = nullptr; t.w = reinterpret_cast<const int8_t*>(e->tw[b]); t.ab = e->tab[b];
    t.gd = e->tgd[b]; t.out = e->arena[(b + 1) % 2]; t.err = e->err;
    t.G0 = G0; t.G = Gt; t.N = e->n; t.H = e->h[b]; t.W = e->w[b]; t.prologue_f16 = e->trans_f16[b];
    t.tile_groups = Gt;
    t.out_tile_groups = e->c0[b + 1] / 32 + e->L[b + 1];
    return dn8::launch_trans(t, e->sms, st, pdl);
}

// One pass of up to n_cap images (images [0, n) of the pass are real), through dense block
// `last_block`: its transition (or, for the last block, the pooling + head) runs only when the pass
// goes past it.
static int engine_pass(dn8_engine* e, const dn8_input* in, int img0, int n, float* feat, float* logits,
                       float* view_logits, int per_view, cudaStream_t st, int last_block = 1 << 30) {
    const int cap = e->n;
    cudaError_t ce;
    // stem -> block 0 input groups (arena 0)
    {
        dn8_stem_args s{};
        const size_t img_elems = static_cast<size_t>(3) * e->img * e->img;
        s.x = in->x_u8 ? in->x : static_cast<const void*>(static_cast<const uint16_t*>(in->x) + img_elems * img0);
        s.src = in->x_u8 ? in->src + static_cast<size_t>(img0) * 4 : nullptr;
        s.flags = in->flags ? in->flags + img0 : nullptr;
        s.w = reinterpret_cast<const int8_t*>(e->sw); s.kc = e->kc; s.out = e->arena[0]; s.err = e->err;
        s.N = n; s.H = e->img; s.W = e->img; s.x_u8 = in->x_u8; s.n_alloc = cap;
        s.tile_groups = e->c0[0] / 32 + e->L[0];
        if ((ce = dn8::launch_stem(s, e->sms, st)) != cudaSuccess) return efail(e, DN8_ECUDA, "stem: %s", cudaGetErrorString(ce));
        mark(e, DN8_K_STEM, 0, 0, st);
    }
    for (int b = 0; b < e->n_blocks && b <= last_block; ++b) {
        const int HW = e->h[b] * e->w[b], G0 = e->c0[b] / 32, Gt = G0 + e->L[b];
        for (int l = 0; l < e->L[b]; ++l) {
            if ((ce = launch_conv1_of(e, b, l, st, true)) != cudaSuccess)
                return efail(e, DN8_ECUDA, "conv1 b%d l%d: %s", b, l, cudaGetErrorString(ce));
            mark(e, DN8_K_CONV1, b, l, st);
            if ((ce = launch_conv2_of(e, b, l, st, true)) != cudaSuccess)
                return efail(e, DN8_ECUDA, "conv2 b%d l%d: %s", b, l, cudaGetErrorString(ce));
            mark(e, DN8_K_CONV2, b, l, st);
        }
        if (b == last_block) break;
        if (e->trans[b]) {
            if ((ce = launch_trans_of(e, b, st, true)) != cudaSuccess)
                return efail(e, DN8_ECUDA, "transition %d: %s", b, cudaGetErrorString(ce));
            mark(e, DN8_K_TRANS, b, 0, st);
        } else {
            dn8_head_args hd{};
            hd.in0 = e->arena[b % 2]; hd.seg = nullptr; hd.fab = e->fab;
            hd.tile_groups = Gt;
            const int C = Gt * 32;
            hd.feat = feat ? feat + static_cast<size_t>(img0) * C : nullptr;
            hd.hw = e->hw; hd.hb = e->hb;
            hd.logits = (e->hw && logits) ? logits + static_cast<size_t>(img0) * e->n_out : nullptr;
            if (hd.logits == nullptr) hd.hw = nullptr;
            hd.view_logits = (hd.hw && view_logits && per_view > 0) ? view_logits + static_cast<size_t>(img0 / per_view) * e->n_out : nullptr;
            hd.tickets = e->tickets;
            hd.G0 = G0; hd.G = Gt; hd.N = n; hd.HW = HW; hd.n_out = e->n_out; hd.per_view = per_view;
            hd.n_alloc = cap;
            if ((ce = dn8::launch_head(hd, st, true)) != cudaSuccess) return efail(e, DN8_ECUDA, "head: %s", cudaGetErrorString(ce));
            mark(e, DN8_K_HEAD, b, 0, st);
        }
    }
    return DN8_OK;
}

int dn8_engine_forward_to(dn8_engine* e, const dn8_input* in, int32_t n, int32_t last_block, dn8_stream stream) {
    if (e == nullptr || in == nullptr || in->x == nullptr || n < 1 || n > e->n || last_block < 0 ||
        last_block >= e->n_blocks || (in->x_u8 && in->src == nullptr))
        return efail(e, DN8_EINVAL, "forward_to: bad arguments (n must fit one pass, 0 <= last_block < %d)",
                     e ? e->n_blocks : 0);
    int prev = 0;
    cudaGetDevice(&prev);
    if (prev != e->device) cudaSetDevice(e->device);
    const int rc = engine_pass(e, in, 0, n, nullptr, nullptr, nullptr, 0, static_cast<cudaStream_t>(stream), last_block);
    if (prev != e->device) cudaSetDevice(prev);
    return rc;
}

int dn8_engine_launch(dn8_engine* e, int32_t kind, int32_t block, int32_t layer, dn8_stream stream) {
    if (e == nullptr || block < 0 || block >= e->n_blocks ||
        !((kind == DN8_K_CONV1 || kind == DN8_K_CONV2) ? layer >= 0 && layer < e->L[block]
                                                       : kind == DN8_K_TRANS && e->trans[block]))
        return efail(e, DN8_EINVAL, "launch: no kernel of kind %d at block %d layer %d", kind, block, layer);
    int prev = 0;
    cudaGetDevice(&prev);
    if (prev != e->device) cudaSetDevice(e->device);
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    const cudaError_t ce = kind == DN8_K_CONV1 ? launch_conv1_of(e, block, layer, st, false)
                         : kind == DN8_K_CONV2 ? launch_conv2_of(e, block, layer, st, false)
                                               : launch_trans_of(e, block, st, false);
    if (prev != e->device) cudaSetDevice(prev);
    return ce == cudaSuccess ? DN8_OK : efail(e, DN8_ECUDA, "launch: %s", cudaGetErrorString(ce));
}

int dn8_engine_forward(dn8_engine* e, const dn8_input* in, int32_t n, float* feat, float* logits,
                       float* view_logits, int32_t per_view, dn8_stream stream) {
    if (e == nullptr || in == nullptr || in->x == nullptr || n < 1) return efail(e, DN8_EINVAL, "forward: bad arguments");
    if (in->x_u8 && in->src == nullptr) return efail(e, DN8_EINVAL, "forward: uint8 planes need a plane table");
    if (view_logits && (per_view < 1 || n % per_view || e->n % per_view))
        return efail(e, DN8_EINVAL, "forward: per_view %d must divide n (%d) and the pass size (%d)", per_view, n, e->n);
    int prev = 0;
    cudaGetDevice(&prev);
    if (prev != e->device) cudaSetDevice(e->device);
    int rc = DN8_OK;
    for (int img0 = 0; img0 < n && rc == DN8_OK; img0 += e->n)
        rc = engine_pass(e, in, img0, std::min(e->n, n - img0), feat, logits, view_logits, per_view,
                         static_cast<cudaStream_t>(stream));
    if (prev != e->device) cudaSetDevice(prev);
    return rc;
}

int dn8_engine_profile(dn8_engine* e, const dn8_input* in, int32_t n, float* feat, dn8_launch_info* out,
                       int32_t max_out, int32_t* n_launches, dn8_stream stream) {
    if (e == nullptr || in == nullptr || out == nullptr || n_launches == nullptr || n < 1 || n > e->n)
        return efail(e, DN8_EINVAL, "profile: bad arguments (n must fit one pass)");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    int prev = 0;
    cudaGetDevice(&prev);
    if (prev != e->device) cudaSetDevice(e->device);
    if (e->events.empty()) {
        e->events.resize(512);
        for (cudaEvent_t& ev : e->events) cudaEventCreate(&ev);
    }
    e->rec.clear();
    e->profiling = true;
    cudaEventRecord(e->events[0], st);
    int rc = engine_pass(e, in, 0, n, feat, nullptr, nullptr, 0, st);
    e->profiling = false;
    cudaError_t ce = cudaStreamSynchronize(st);
    if (rc == DN8_OK && ce != cudaSuccess) rc = efail(e, DN8_ECUDA, "profile: %s", cudaGetErrorString(ce));
    int k = 0;
    for (; rc == DN8_OK && k < static_cast<int>(e->rec.size()) && k < max_out; ++k) {
        float ms = 0.0f;
        cudaEventElapsedTime(&ms, e->events[k], e->events[k + 1]);
        out[k] = e->rec[k];
        out[k].ms = ms;
    }
    *n_launches = k;
    if (prev != e->device) cudaSetDevice(prev);
    return rc;
}

int dn8_engine_check(dn8_engine* e, dn8_stream stream) {
    if (e == nullptr) return DN8_EINVAL;
    int32_t code = 0;
    cudaError_t ce = cudaMemcpyAsync(&code, e->err, 4, cudaMemcpyDeviceToHost, static_cast<cudaStream_t>(stream));
    if (ce == cudaSuccess) ce = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
    if (ce != cudaSuccess) return efail(e, DN8_ECUDA, "check: %s", cudaGetErrorString(ce));
    if (code != 0) {
        cudaMemsetAsync(e->err, 0, 4, static_cast<cudaStream_t>(stream));
        cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
        return efail(e, DN8_EDEVICE, "a kernel gave up a bounded wait (code %d)", code);
    }
    return DN8_OK;
}

}  // extern "C"

// The engine's tile-major stores hold q + 128 per byte (offset binary): the copied segment is flipped
// back to signed q in place, on the device, or on the host once the copy has landed.
__global__ void store_to_signed_kernel(uint8_t* p, size_t n) {
    for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<size_t>(gridDim.x) * blockDim.x)
        p[i] ^= 0x80u;
}
struct HostFlip {
    uint8_t* p;
    size_t n;
};
static void CUDART_CB host_to_signed(void* arg) {
    HostFlip* f = static_cast<HostFlip*>(arg);
    for (size_t i = 0; i < f->n; ++i) f->p[i] ^= 0x80u;
    delete f;
}

extern "C" {

int dn8_engine_store(const dn8_engine* ec, int32_t block, int32_t j, int8_t* dst, dn8_stream stream) {
    dn8_engine* e = const_cast<dn8_engine*>(ec);
    if (e == nullptr || block < 0 || block >= e->n_blocks || j < 0 || j > e->L[block] || dst == nullptr)
        return efail(e, DN8_EINVAL, "store: bad arguments");
    const size_t rows = static_cast<size_t>(e->n) * e->h[block] * e->w[block];
    const size_t full = rows / 128, rest = rows % 128;             // whole tiles, rows of the last one
    const int G0 = e->c0[block] / 32, Gt = G0 + e->L[block];
    const int8_t* base = e->arena[block % 2];
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    // group g of the tile-major store [tiles][Gt][128][32] -> rows x 32 bytes at dst, per group:
    // the whole tiles as one strided copy (4 KB per tile, Gt * 4 KB apart), then the partial last tile
    cudaError_t ce = cudaSuccess;
    const int g0 = j == 0 ? 0 : G0 + j - 1, ng = j == 0 ? G0 : 1;
    for (int g = g0; g < g0 + ng && ce == cudaSuccess; ++g) {
        int8_t* d = dst + static_cast<size_t>(g - g0) * rows * 32;
        const int8_t* sg = base + static_cast<size_t>(g) * 4096;
        if (full > 0)
            ce = cudaMemcpy2DAsync(d, 4096, sg, static_cast<size_t>(Gt) * 4096, 4096, full, cudaMemcpyDefault, st);
        if (ce == cudaSuccess && rest > 0)
            ce = cudaMemcpyAsync(d + full * 4096, sg + full * Gt * 4096, rest * 32, cudaMemcpyDefault, st);
    }
    if (ce == cudaSuccess) {
        const size_t bytes = static_cast<size_t>(ng) * rows * 32;
        cudaPointerAttributes pa{};
        ce = cudaPointerGetAttributes(&pa, dst);
        if (ce == cudaSuccess && (pa.type == cudaMemoryTypeDevice || pa.type == cudaMemoryTypeManaged)) {
            store_to_signed_kernel<<<e->sms, 256, 0, st>>>(reinterpret_cast<uint8_t*>(dst), bytes);
            ce = cudaGetLastError();
        } else if (ce == cudaSuccess) {
            HostFlip* f = new (std::nothrow) HostFlip{reinterpret_cast<uint8_t*>(dst), bytes};
            ce = f == nullptr ? cudaErrorMemoryAllocation : cudaLaunchHostFunc(st, host_to_signed, f);
            if (ce != cudaSuccess) delete f;
        }
    }
    return ce == cudaSuccess ? DN8_OK : efail(e, DN8_ECUDA, "store: %s", cudaGetErrorString(ce));
}

}  // extern "C"
