// zoom.cu -- the geometric test-time view in front of the stem: zoom `scale` about the centre and
// shift (tx, ty) (fractions of the side) of every slice-triplet window, bilinear, zero outside,
// written as the fp16 windows the stem's fp16 path reads. Restates the reference's `affine_windows`
// (src/knee/tta.py:131-149: `affine_grid` + `grid_sample`, bilinear, zeros, align_corners=False, in
// fp16) with the pixels gathered straight from the uint8 volume planes (the reference's
// `gather_u8_to_f16` LUT, src/knee/data/fused_uint8.py:735: fp16(u * fp32(1/255))) and an optional
// horizontal flip of the source window.
//
// Arithmetic, per output pixel (x, y) of a W x H window:
//   base grid   bx = fp16(fp16(l_x * (W - 1)) / W), l_x = the fp16 linspace(-1, 1, W) element
//               (start + step i below the middle, end - step (W - 1 - i) from it, in fp16);
//   grid        gx = fp16(fp32(t00 bx + t02)), t00 = fp16(1 / scale), t02 = fp16(-2 tx) (the
//               3-term dot product of affine_grid, exact products, one fp32 sum);
//   source      ix = ((gx + 1) W - 1) / 2, corners floor(ix) (+1), bilinear weights as products of
//               the distances, accumulated nw, ne, sw, se with fmaf in fp32, then rounded to fp16.
#include "dn8_common.cuh"
#include "dn8_kernels.h"

namespace dn8 {

constexpr int ZM_THREADS = 256;

// fp16 rounding of an fp32 value, returned as fp32
DN8_DEV float f16r(float v) { return __half2float(__float2half_rn(v)); }

// base-grid coordinate i of n points (align_corners = False): the fp16 linspace(-1, 1, n) element
// in fp16 arithmetic (step = fp16(2 / (n - 1)); -1 + step i below the middle, 1 - step (n - 1 - i)
// from it, each product and sum rounded to fp16), scaled by (n - 1) / n as two fp16-rounded steps
DN8_DEV float base_coord(int i, int n, __half step) {
    if (n <= 1) return 0.0f;
    // (the _rn forms: a product and a sum, never contracted into one fma)
    const __half l = (i < n / 2) ? __hadd_rn(__float2half_rn(-1.0f), __hmul_rn(step, __int2half_rn(i)))
                                 : __hsub_rn(__float2half_rn(1.0f), __hmul_rn(step, __int2half_rn(n - 1 - i)));
    return f16r(f16r(__half2float(l) * static_cast<float>(n - 1)) / static_cast<float>(n));
}

// One CTA = a band of ZM_ROWS output rows of one (image, channel) window. The source rows the band
// samples (a contiguous range, zoom-dependent) are staged in shared memory as fp32 pixel values
// (the fp16 LUT value of each byte) with 16-byte loads; the column terms (source columns after the
// optional mirror, weights) and the row terms are computed once per CTA. A tap outside the window
// gets weight 0 and a valid address: fmaf(v, 0, acc) = acc exactly (v >= 0), which is the reference's
// "skip the tap". Each thread then writes pairs of adjacent fp16 outputs.
constexpr int ZM_ROWS = 16;

DN8_DEV float src_coord(int i, int n, float t00, float t02, __half step) {
    const float g = f16r(t00 * base_coord(i, n, step) + t02);
    return ((g + 1.0f) * static_cast<float>(n) - 1.0f) * 0.5f;
}

__global__ void __launch_bounds__(ZM_THREADS) zoom_kernel(const dn8_zoom_args a, float t00, float t02x, float t02y,
                                                          __half stepx, __half stepy, int max_src_rows) {
    extern __shared__ __align__(16) uint8_t zsm[];
    const int H = a.H, W = a.W;
    float4* ctab = reinterpret_cast<float4*>(zsm);              // [W] (source col x0, x0 + 1, w0, w1)
    float4* rtab = ctab + W;                                    // [ZM_ROWS] (row off 0, 1, w0, w1)
    float* fsrc = reinterpret_cast<float*>(rtab + ZM_ROWS);     // [max_src_rows][W] staged pixels
    const int bands = (H + ZM_ROWS - 1) / ZM_ROWS;
    const int band = static_cast<int>(blockIdx.x % bands);
    const int plane_idx = static_cast<int>(blockIdx.x / bands);    // n * 3 + ch
    const int n = plane_idx / 3, ch = plane_idx - 3 * n;
    const int yb = band * ZM_ROWS, ye = min(H, yb + ZM_ROWS);
    const int flip = a.flags != nullptr ? (a.flags[n] & 1) : 0;
    const uint8_t* plane = a.planes + static_cast<size_t>(a.src[n * 4 + ch]) * H * W;
    // source rows [r0, r0 + nr) cover floor(iy) .. floor(iy) + 1 of every row of the band
    const int r0 = static_cast<int>(floorf(src_coord(yb, H, t00, t02y, stepy)));
    const int r1 = static_cast<int>(floorf(src_coord(ye - 1, H, t00, t02y, stepy))) + 1;
    const int nr = r1 - r0 + 1;
    if (nr > max_src_rows) {                                    // cannot happen for scale >= 0.25
        if (threadIdx.x == 0 && a.err != nullptr) atomicCAS(a.err, 0, ERR_SHAPE);
        return;
    }
    for (int k = threadIdx.x; k < nr * (W >> 4); k += ZM_THREADS) {
        const int r = k / (W >> 4), c16 = k - r * (W >> 4);
        const int yy = r0 + r;
        uint4 v = make_uint4(0u, 0u, 0u, 0u);
        if (yy >= 0 && yy < H) v = __ldg(reinterpret_cast<const uint4*>(plane + static_cast<size_t>(yy) * W) + c16);
        const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
        float* d = fsrc + r * W + 16 * c16;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            float4 f;
            // the reference's LUT: fp16(u * fp32(1 / 255))
            f.x = f16r(static_cast<float>(w4[q] & 0xFFu) * (1.0f / 255.0f));
            f.y = f16r(static_cast<float>((w4[q] >> 8) & 0xFFu) * (1.0f / 255.0f));
            f.z = f16r(static_cast<float>((w4[q] >> 16) & 0xFFu) * (1.0f / 255.0f));
            f.w = f16r(static_cast<float>(w4[q] >> 24) * (1.0f / 255.0f));
            reinterpret_cast<float4*>(d)[q] = f;
        }
    }
    for (int x = threadIdx.x; x < W; x += ZM_THREADS) {
        const float ix = src_coord(x, W, t00, t02x, stepx);
        const float fx0 = floorf(ix);
        const int x0 = static_cast<int>(fx0), x1 = x0 + 1;
        float w0 = (fx0 + 1.0f) - ix, w1 = ix - fx0;
        const bool v0 = x0 >= 0 && x0 < W, v1 = x1 >= 0 && x1 < W;
        int s0 = flip ? W - 1 - x0 : x0, s1 = flip ? W - 1 - x1 : x1;   // the (mirrored) window
        if (!v0) { s0 = 0; w0 = 0.0f; }
        if (!v1) { s1 = 0; w1 = 0.0f; }
        ctab[x] = make_float4(__int_as_float(s0), __int_as_float(s1), w0, w1);
    }
    if (threadIdx.x < ye - yb) {
        const float iy = src_coord(yb + threadIdx.x, H, t00, t02y, stepy);
        const float fy0 = floorf(iy);
        const int y0 = static_cast<int>(fy0);
        float w0 = (fy0 + 1.0f) - iy, w1 = iy - fy0;
        int o0 = (y0 - r0) * W, o1 = o0 + W;
        if (!(y0 >= 0 && y0 < H)) { o0 = 0; w0 = 0.0f; }
        if (!(y0 + 1 >= 0 && y0 + 1 < H)) { o1 = 0; w1 = 0.0f; }
        rtab[threadIdx.x] = make_float4(__int_as_float(o0), __int_as_float(o1), w0, w1);
    }
    __syncthreads();
    const int pairs = W >> 1;
    for (int k = threadIdx.x; k < (ye - yb) * pairs; k += ZM_THREADS) {
        const int yl = k / pairs, x = 2 * (k - yl * pairs);
        const float4 rt = rtab[yl];
        const float* row0 = fsrc + __float_as_int(rt.x);
        const float* row1 = fsrc + __float_as_int(rt.y);
        float o[2];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
            const float4 ct = ctab[x + e];
            const int s0 = __float_as_int(ct.x), s1 = __float_as_int(ct.y);
            float acc = 0.0f;
            acc = fmaf(row0[s0], ct.z * rt.z, acc);             // nw, ne, sw, se as the reference
            acc = fmaf(row0[s1], ct.w * rt.z, acc);
            acc = fmaf(row1[s0], ct.z * rt.w, acc);
            acc = fmaf(row1[s1], ct.w * rt.w, acc);
            o[e] = acc;
        }
        __half* out = reinterpret_cast<__half*>(a.out) + (static_cast<size_t>(plane_idx) * H + yb + yl) * W;
        *reinterpret_cast<__half2*>(out + x) = __floats2half2_rn(o[0], o[1]);
    }
}

static int zoom_src_rows(double scale) {
    // rows a band of ZM_ROWS output rows samples: about ZM_ROWS / scale, plus the two ends
    return static_cast<int>(ZM_ROWS / scale) + 4;
}

static size_t zoom_smem(int W, int src_rows) {
    return static_cast<size_t>(W) * 16 + ZM_ROWS * 16 + static_cast<size_t>(src_rows) * W * 4;
}

cudaError_t launch_zoom(const dn8_zoom_args& a, int sms, cudaStream_t st) {
    (void)sms;
    // the theta entries are rounded to fp16 from double, as a Python float in an fp16 tensor
    const float t00 = __half2float(__double2half(1.0 / a.scale));
    const float t02x = __half2float(__double2half(-2.0 * a.tx));
    const float t02y = __half2float(__double2half(-2.0 * a.ty));
    if (a.W % 16 || a.scale < 0.25) return cudaErrorInvalidValue;
    const int src_rows = zoom_src_rows(a.scale);
    const size_t smem = zoom_smem(a.W, src_rows);
    if (smem > 227 * 1024) return cudaErrorInvalidValue;
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(zoom_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (e != cudaSuccess) return e;
    }
    const long long blocks = static_cast<long long>(a.N) * 3 * ((a.H + ZM_ROWS - 1) / ZM_ROWS);
    if (blocks <= 0) return cudaSuccess;
    if (blocks > 0x7FFFFFFFLL) return cudaErrorInvalidValue;
    const __half stepx = __double2half(2.0 / static_cast<double>(a.W - 1));
    const __half stepy = __double2half(2.0 / static_cast<double>(a.H - 1));
    return launch_pdl(false, zoom_kernel, dim3(static_cast<unsigned>(blocks)), dim3(ZM_THREADS), smem, st, a, t00, t02x,
                      t02y, stepx, stepy, src_rows);
}

}  // namespace dn8
