/* dn8_oracle.c -- TEST INFRASTRUCTURE ONLY: a CPU restatement of the reference INT8 DenseNet
 * arithmetic, used by tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg as the
 * checker. Nothing in the product (rsna_knee_efficiency_b200/) links, imports or calls it.
 *
 * Two arithmetic modes for every operator:
 *   ORC_KERNEL  (0): the reference CUDA kernels' fp32 arithmetic (src/knee/dense8s_kernels.cu):
 *                    fp32 fmaf epilogues, rint via the 2^23 / 1.5*2^23 adds, fp16 prologue
 *                    `pro4h` (:122-139), fp32 prologue `pro16` (:99-120), conv1 epilogue
 *                    (:598-611), conv2 epilogue (:2797-2810), integer transition (:375-389),
 *                    `stem_i8` epilogue + byte max-pool (:3734-3767), `final_q` (:2306-2323).
 *                    The GPU kernels of this repository must match this mode byte for byte.
 *   ORC_EMULATE (1): the float64 fake-quant emulation `dense8s.emulate` / `stem_q_i8`
 *                    (src/knee/dense8s.py:549-643). Pinned against golden vectors produced by
 *                    the reference itself (tests/golden/).
 * The integer accumulators are exact (int32 / int64) in both modes.
 *
 * Layouts (channel-last): a block store X is int8 [P][C] with P = N*H*W pixels; the u8 bottleneck
 * is [P][128]; the stem input is [N][3][H][W] (u8 bytes, or fp16 bits); outputs likewise.
 * Build: oracle/Makefile (gcc -O2 -ffp-contract=off, OpenMP over pixels).
 */
#include <math.h>
#include <stdint.h>
#include <string.h>
#include <stdlib.h>

#define ORC_KERNEL 0
#define ORC_EMULATE 1

/* ---- scalar helpers ---------------------------------------------------------------------- */
static inline float bits_f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static inline uint32_t f_bits(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }

static inline float sat01f(float x) { return x > 0.f ? (x < 1.f ? x : 1.f) : 0.f; } /* NaN -> 0 */
static inline double clampd(double x, double lo, double hi) { return x < lo ? lo : (x > hi ? hi : x); }

/* fp16 bits -> double (exact). */
static double f16_to_d(uint16_t h) {
    int s = h >> 15, e = (h >> 10) & 31, m = h & 1023;
    double v;
    if (e == 0) v = ldexp((double)m, -24);
    else if (e == 31) v = m ? NAN : INFINITY;
    else v = ldexp((double)(m | 1024), e - 25);
    return s ? -v : v;
}

/* double -> fp16 value (as double), round to nearest even, overflow to inf. */
static double d_to_f16d(double x) {
    if (x != x) return x;
    double a = fabs(x);
    if (a >= 65520.0) return x > 0 ? INFINITY : -INFINITY;
    int e;
    frexp(a, &e);                      /* a = f * 2^e, f in [0.5, 1) */
    int ulp_e = e - 11;                /* 11 significant bits */
    if (ulp_e < -24) ulp_e = -24;      /* subnormal spacing */
    double q = ldexp(a, -ulp_e);
    double r = nearbyint(q);           /* default rounding mode: to nearest even */
    double v = ldexp(r, ulp_e);
    return x < 0 ? -v : v;
}

/* u = rint(255 v) through fmaf(v, 255, 2^23): the low byte of the float. */
static inline uint8_t u8_of_unit(float v) { return (uint8_t)(f_bits(fmaf(v, 255.0f, 8388608.0f)) & 0xFFu); }
/* q = rint(t) for t in [-127, 127] through t + 1.5 * 2^23. */
static inline int8_t s8_of_f(float t) { return (int8_t)(f_bits(t + 12582912.0f) & 0xFFu); }

/* ---- prologue: store byte q -> u8 u for channel c ------------------------------------------ */
/* ab: [C][2] float (fp32 prologue) or NULL; abh: [C/2][4] fp16 bits (A_2p, A_2p+1, B_2p, B_2p+1). */
static inline uint8_t prologue(int8_t q, int c, const float* ab, const uint16_t* abh, int mode) {
    if (abh) {
        const uint16_t* p = abh + (c >> 1) * 4;
        double A = f16_to_d(p[c & 1]), B = f16_to_d(p[2 + (c & 1)]);
        /* fp16 fma(A, q, B): the exact value (representable in double for fp16 operands) rounded
         * once to fp16, saturated to [0, 1]; u = rint(255 v). Identical in both modes. */
        double t = A * (double)q + B;
        double v = d_to_f16d(t);
        v = v > 0.0 ? (v < 1.0 ? v : 1.0) : 0.0;
        return (uint8_t)nearbyint(v * 255.0);
    }
    const float a = ab[2 * c], b = ab[2 * c + 1];
    if (mode == ORC_KERNEL) {
        return u8_of_unit(sat01f(fmaf(a, (float)q, b)));
    } else {
        double t = (double)a * (double)q + (double)b;
        t = clampd(t, 0.0, 1.0);
        return (uint8_t)nearbyint(t * 255.0);
    }
}

/* ---- conv1: X int8 [P][cin] -> u8 bottleneck [P][128] ------------------------------------------
 * acc[o] = sum_c W[o][c] u_c (exact), W from the chunked pack table w1c [cin/32][128][32];
 * out = rint(255 sat(g acc + d)), gd [128][2]. acc_out (optional) [P][128] int32.
 * Reference: conv1w_body `dense8s_kernels.cu:479-627`; emulate `dense8s.py:578-591`. */
void orc_conv1(const int8_t* X, long P, int cin, const int8_t* w1c, const float* ab,
               const uint16_t* abh, const float* gd, int mode, uint8_t* out, int32_t* acc_out) {
    const int G = cin / 32;
    int8_t* W = (int8_t*)malloc((size_t)128 * cin);
    for (int g = 0; g < G; ++g)
        for (int o = 0; o < 128; ++o)
            for (int i = 0; i < 32; ++i) W[(size_t)o * cin + g * 32 + i] = w1c[((size_t)g * 128 + o) * 32 + i];
    #pragma omp parallel
    {
        uint8_t* u = (uint8_t*)malloc(cin);
        int32_t* ui = (int32_t*)malloc(sizeof(int32_t) * cin);
        #pragma omp for schedule(static)
        for (long p = 0; p < P; ++p) {
            const int8_t* x = X + p * cin;
            for (int c = 0; c < cin; ++c) { u[c] = prologue(x[c], c, ab, abh, mode); ui[c] = u[c]; }
            for (int o = 0; o < 128; ++o) {
                const int8_t* w = W + (size_t)o * cin;
                int32_t acc = 0;
                for (int c = 0; c < cin; ++c) acc += (int32_t)w[c] * ui[c];
                if (acc_out) acc_out[p * 128 + o] = acc;
                const float g = gd[2 * o], d = gd[2 * o + 1];
                uint8_t r;
                if (mode == ORC_KERNEL) {
                    r = u8_of_unit(sat01f(fmaf(g, (float)acc, d)));
                } else {
                    double t = (double)g * (double)acc + (double)d;
                    r = (uint8_t)nearbyint(clampd(t, 0.0, 1.0) * 255.0);
                }
                out[p * 128 + o] = r;
            }
        }
        free(u);
        free(ui);
    }
    free(W);
}

/* ---- conv2: u8 [N][H][W][128] -> int8 [N][H][W][32], 3x3 pad 1 --------------------------------
 * acc = sum_{blk,tap,i} w2k[blk][tap][o][i] v (zero padding); q = rint(clamp(acc sc_o, +-127)).
 * Reference: conv2t_body `dense8s_kernels.cu:2679-2832`; emulate `dense8s.py:592-599`. */
void orc_conv2(const uint8_t* V, int N, int H, int Wd, const int8_t* w2k, const float* sc, int mode,
               int8_t* out, int32_t* acc_out) {
    const long P = (long)N * H * Wd;
    #pragma omp parallel for schedule(static)
    for (long p = 0; p < P; ++p) {
        const int n = (int)(p / ((long)H * Wd));
        const int rem = (int)(p - (long)n * H * Wd), y = rem / Wd, x = rem % Wd;
        int32_t acc[32];
        for (int o = 0; o < 32; ++o) acc[o] = 0;
        for (int tap = 0; tap < 9; ++tap) {
            const int yy = y + tap / 3 - 1, xx = x + tap % 3 - 1;
            if (yy < 0 || yy >= H || xx < 0 || xx >= Wd) continue;
            const uint8_t* v = V + (((long)n * H + yy) * Wd + xx) * 128;
            for (int blk = 0; blk < 4; ++blk)
                for (int o = 0; o < 32; ++o) {
                    const int8_t* w = w2k + (((size_t)blk * 9 + tap) * 32 + o) * 32;
                    int32_t s = 0;
                    for (int i = 0; i < 32; ++i) s += (int32_t)w[i] * (int32_t)v[blk * 32 + i];
                    acc[o] += s;
                }
        }
        for (int o = 0; o < 32; ++o) {
            if (acc_out) acc_out[p * 32 + o] = acc[o];
            int8_t r;
            if (mode == ORC_KERNEL) {
                float t = (float)acc[o] * sc[o];
                t = fminf(fmaxf(t, -127.0f), 127.0f);
                r = s8_of_f(t);
            } else {
                double t = nearbyint((double)acc[o] * (double)sc[o]);
                r = (int8_t)clampd(t, -127.0, 127.0);
            }
            out[p * 32 + o] = r;
        }
    }
}

/* ---- transition: X int8 [N][H][W][C] -> int8 [N][H/2][W/2][C/2] --------------------------------
 * u = prologue; acc = 1x1 conv (exact); s = sum of the 2x2 square's four accumulators (exact);
 * q = rint(clamp(k_o s, +-127)), k = T_gd[o][0]. The integer form `gemm_q<.., MODE 1>`
 * (`dense8s_kernels.cu:375-389`) and emulate's `avg_pool2d(acc, 2) * 4` (`dense8s.py:601-615`). */
void orc_trans(const int8_t* X, int N, int H, int Wd, int C, const int8_t* wc, const float* ab,
               const uint16_t* abh, const float* gd, int mode, int8_t* out) {
    const int G = C / 32, cout = C / 2, H2 = H / 2, W2 = Wd / 2;
    int8_t* Wt = (int8_t*)malloc((size_t)cout * C);
    for (int g = 0; g < G; ++g)
        for (int o = 0; o < cout; ++o)
            for (int i = 0; i < 32; ++i) Wt[(size_t)o * C + g * 32 + i] = wc[((size_t)g * cout + o) * 32 + i];
    const long PO = (long)N * H2 * W2;
    #pragma omp parallel
    {
        int32_t* u4 = (int32_t*)malloc(sizeof(int32_t) * 4 * C);
        #pragma omp for schedule(static)
        for (long po = 0; po < PO; ++po) {
            const int n = (int)(po / ((long)H2 * W2));
            const int rem = (int)(po - (long)n * H2 * W2), oy = rem / W2, ox = rem % W2;
            for (int k = 0; k < 4; ++k) {
                const int y = 2 * oy + (k >> 1), x = 2 * ox + (k & 1);
                const int8_t* xp = X + (((long)n * H + y) * Wd + x) * C;
                for (int c = 0; c < C; ++c) u4[k * C + c] = prologue(xp[c], c, ab, abh, mode);
            }
            for (int o = 0; o < cout; ++o) {
                const int8_t* w = Wt + (size_t)o * C;
                int64_t s = 0;
                for (int k = 0; k < 4; ++k) {
                    int32_t acc = 0;
                    for (int c = 0; c < C; ++c) acc += (int32_t)w[c] * u4[k * C + c];
                    s += acc;
                }
                const float kk = gd[2 * o];
                int8_t r;
                if (mode == ORC_KERNEL) {
                    float t = fminf(fmaxf(kk * (float)(int32_t)s, -127.0f), 127.0f);
                    r = s8_of_f(t);
                } else {
                    double t = nearbyint((double)kk * (double)s);
                    r = (int8_t)clampd(t, -127.0, 127.0);
                }
                out[po * cout + o] = r;
            }
        }
        free(u4);
    }
    free(Wt);
}

/* ---- final features: X int8 [N][HW][C] -> float [N][C] -----------------------------------------
 * kernel: four fp32 partial sums over pixels s = q, q+4, ... of relu(fmaf(a, q, b)), then
 * (p0 + p1 + p2 + p3) / HW (`final_q`, `dense8s_kernels.cu:2306-2323`).
 * emulate: relu(a x + b) in float64, mean over the pixels, cast to float (`dense8s.py:616-619`). */
void orc_final(const int8_t* X, int N, int HW, int C, const float* fab, int mode, float* out) {
    #pragma omp parallel for schedule(static)
    for (long nc = 0; nc < (long)N * C; ++nc) {
        const int n = (int)(nc / C), c = (int)(nc % C);
        const float a = fab[2 * c], b = fab[2 * c + 1];
        const int8_t* x = X + (long)n * HW * C + c;
        if (mode == ORC_KERNEL) {
            float part[4];
            for (int q = 0; q < 4; ++q) {
                float acc = 0.f;
                for (int s = q; s < HW; s += 4) acc += fmaxf(fmaf(a, (float)x[(long)s * C], b), 0.f);
                part[q] = acc;
            }
            out[nc] = (part[0] + part[1] + part[2] + part[3]) / (float)HW;
        } else {
            double acc = 0.0;
            for (int s = 0; s < HW; ++s) {
                double z = (double)a * (double)x[(long)s * C] + (double)b;
                acc += z > 0.0 ? z : 0.0;
            }
            out[nc] = (float)(acc / (double)HW);
        }
    }
}

/* ---- stem: [N][3][H][W] pixels -> int8 [N][H/4][W/4][64] (block-1 input, values 0..127) ------
 * u = the u8 byte (in_u8 = 1) or rint(255 sat(x)) of an fp16 pixel (in_u8 = 0); flip = 1 reads
 * column W-1-x. acc = exact 7x7/2 pad-3 conv with the int8 weights w8f [64][3][7][7];
 * kernel: q = rint(clamp(fmaf(acc, k, c), 0, 127)); emulate: q = rint(clamp(fp32(acc k + c), 0, 127))
 * (`stem_i8_body` `dense8s_kernels.cu:3641-3771`, `stem_q_i8` `dense8s.py:625-643`);
 * then a 3x3/2 pad-1 max-pool (out-of-image positions excluded). */
void orc_stem(const void* x, int in_u8, const int* flip, int N, int H, int Wd, const float* w8f,
              const float* kc, int mode, int8_t* out) {
    const int CH = H / 2, CW = Wd / 2, PH = H / 4, PW = Wd / 4;
    int8_t* W8 = (int8_t*)malloc(64 * 147);
    for (int i = 0; i < 64 * 147; ++i) W8[i] = (int8_t)w8f[i];
    #pragma omp parallel
    {
        uint8_t* u = (uint8_t*)malloc((size_t)3 * H * Wd);
        uint8_t* cq = (uint8_t*)malloc((size_t)CH * CW * 64);
        #pragma omp for schedule(static)
        for (int n = 0; n < N; ++n) {
            const int fl = flip ? flip[n] : 0;
            for (int ch = 0; ch < 3; ++ch)
                for (int y = 0; y < H; ++y)
                    for (int xx = 0; xx < Wd; ++xx) {
                        const long src = (((long)n * 3 + ch) * H + y) * Wd + (fl ? Wd - 1 - xx : xx);
                        uint8_t v;
                        if (in_u8) {
                            v = ((const uint8_t*)x)[src];
                        } else {
                            const double a = f16_to_d(((const uint16_t*)x)[src]);
                            if (mode == ORC_KERNEL)
                                v = (uint8_t)(f_bits(fmaf(sat01f((float)a), 255.0f, 12582912.0f)) & 0xFFu);
                            else
                                v = (uint8_t)nearbyint(clampd(a, 0.0, 1.0) * 255.0);
                        }
                        u[((long)ch * H + y) * Wd + xx] = v;
                    }
            for (int cy = 0; cy < CH; ++cy)
                for (int cx = 0; cx < CW; ++cx)
                    for (int o = 0; o < 64; ++o) {
                        int32_t acc = 0;
                        for (int ch = 0; ch < 3; ++ch)
                            for (int ky = 0; ky < 7; ++ky) {
                                const int y = 2 * cy + ky - 3;
                                if (y < 0 || y >= H) continue;
                                for (int kx = 0; kx < 7; ++kx) {
                                    const int xx = 2 * cx + kx - 3;
                                    if (xx < 0 || xx >= Wd) continue;
                                    acc += (int32_t)W8[((o * 3 + ch) * 7 + ky) * 7 + kx] *
                                           (int32_t)u[((long)ch * H + y) * Wd + xx];
                                }
                            }
                        const float k = kc[o], c = kc[64 + o];
                        uint8_t q;
                        if (mode == ORC_KERNEL) {
                            float t = fminf(fmaxf(fmaf((float)acc, k, c), 0.0f), 127.0f);
                            q = (uint8_t)(f_bits(t + 12582912.0f) & 0xFFu);
                        } else {
                            double t = (double)acc * (double)k + (double)c;
                            t = (double)(float)t;
                            q = (uint8_t)nearbyint(clampd(t, 0.0, 127.0));
                        }
                        cq[((long)cy * CW + cx) * 64 + o] = q;
                    }
            for (int py = 0; py < PH; ++py)
                for (int px = 0; px < PW; ++px)
                    for (int o = 0; o < 64; ++o) {
                        uint8_t m = 0;
                        for (int dy = -1; dy <= 1; ++dy) {
                            const int cy = 2 * py + dy;
                            if (cy < 0 || cy >= CH) continue;
                            for (int dx = -1; dx <= 1; ++dx) {
                                const int cx = 2 * px + dx;
                                if (cx < 0 || cx >= CW) continue;
                                const uint8_t v = cq[((long)cy * CW + cx) * 64 + o];
                                if (v > m) m = v;
                            }
                        }
                        out[(((long)n * PH + py) * PW + px) * 64 + o] = (int8_t)m;
                    }
        }
        free(u);
        free(cq);
    }
    free(W8);
}

/* ---- head: features [N][C] -> logits [N][n_out] (fp32, channel order ascending) ----------- */
void orc_head(const float* f, int N, int C, const float* hw, const float* hb, int n_out, float* out) {
    for (int n = 0; n < N; ++n)
        for (int j = 0; j < n_out; ++j) {
            double s = 0.0;
            for (int c = 0; c < C; ++c) s += (double)f[(long)n * C + c] * (double)hw[(long)j * C + c];
            out[n * n_out + j] = (float)(s + (double)hb[j]);
        }
}

int orc_version(void) { return 1; }
