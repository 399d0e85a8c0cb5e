// preprocess.cu -- CLIP image preprocessing on the device.
//
// roofline.c's tc_vit_encode takes pixels already normalised (src/vit.h:75-78)
// and reads the normalisation of the checkpoint from the GGUF
// (clip-vit.preprocess.mean / std, src/vit.c:130-139); its exporter also
// records the resampling filter and the resize rule
// (clip-vit.preprocess.interpolation / resize_mode,
// tools/export_vit_gguf.py:291-294), i.e. open_clip's pipeline: resize the
// shorter side to the image size with PIL, centre crop, scale to [0, 1],
// subtract the mean and divide by the standard deviation.
//
// This file runs that pipeline on decoded 8-bit RGB images (n x height x
// width x 3, interleaved), following PIL's published resampling algorithm
// so that the 8-bit resized pixels are the ones PIL produces:
//   - per output column (row) a window of input columns with filter weights
//     filter((x - centre + 0.5) / max(scale, 1)), support = filter support *
//     max(scale, 1), normalised to sum 1 and rounded to 22-bit fixed point;
//   - a horizontal pass, then a vertical one, each rounding to 8 bits
//     (sum + 2^21, arithmetic shift by 22, clamp to 0..255);
// the coefficient tables are computed on the host in double precision, as
// PIL does. Only the columns and rows inside the centre crop are produced.
// Then x / 255, minus mean, divided by std, in IEEE fp32, planar output.
#include "tcg_common.cuh"

#include <math.h>
#include <string.h>
#include <vector>

namespace tcg {

namespace {

constexpr int PRE_BITS = 22;            // fixed-point precision of the 8-bit passes

// Host: PIL's filters.
double bicubic(double x)
{
    const double a = -0.5;
    if (x < 0.0) x = -x;
    if (x < 1.0) return ((a + 2.0) * x - (a + 3.0)) * x * x + 1.0;
    if (x < 2.0) return (((x - 5.0) * x + 8.0) * x - 4.0) * a;
    return 0.0;
}
double bilinear(double x)
{
    if (x < 0.0) x = -x;
    return x < 1.0 ? 1.0 - x : 0.0;
}

// The taps of output index o of a resize from in_size to out_size: first
// input index, count, and int32 coefficients (ksize slots per output).
struct Axis {
    int ksize = 0;
    std::vector<int> first, count, coef;
};

Axis axis_coeffs(int in_size, int out_size, int interp, int o_begin, int o_count)
{
    const double support0 = interp == 0 ? 2.0 : 1.0;
    const double scale = (double)in_size / (double)out_size;
    const double fscale = scale > 1.0 ? scale : 1.0;
    const double support = support0 * fscale;
    Axis ax;
    ax.ksize = (int)ceil(support) * 2 + 1;
    ax.first.resize(o_count);
    ax.count.resize(o_count);
    ax.coef.assign((size_t)o_count * ax.ksize, 0);
    std::vector<double> k(ax.ksize);
    for (int i = 0; i < o_count; i++) {
        const int o = o_begin + i;
        const double centre = (o + 0.5) * scale;
        const double ss = 1.0 / fscale;
        int xmin = (int)(centre - support + 0.5);
        if (xmin < 0) xmin = 0;
        int xmax = (int)(centre + support + 0.5);
        if (xmax > in_size) xmax = in_size;
        xmax -= xmin;
        double ww = 0.0;
        for (int x = 0; x < xmax; x++) {
            const double t = (x + xmin - centre + 0.5) * ss;
            k[x] = interp == 0 ? bicubic(t) : bilinear(t);
            ww += k[x];
        }
        for (int x = 0; x < xmax; x++) {
            const double w = ww != 0.0 ? k[x] / ww : k[x];
            // round half away from zero to 22-bit fixed point
            ax.coef[(size_t)i * ax.ksize + x] = (int)(w * (double)(1 << PRE_BITS) + (w < 0.0 ? -0.5 : 0.5));
        }
        ax.first[i] = xmin;
        ax.count[i] = xmax;
    }
    return ax;
}

__device__ __forceinline__ unsigned clip8(int v)
{
    v >>= PRE_BITS;                           // arithmetic: floor
    return v < 0 ? 0u : (v > 255 ? 255u : (unsigned)v);
}

// Horizontal pass: tmp[n][y][ox][c] for input rows y0 .. y0+rows-1 and the
// crop's ow output columns.
__global__ void pre_horizontal_kernel(const uint8_t *__restrict__ rgb, uint8_t *__restrict__ tmp, int n, int h, int w,
                                      int y0, int rows, int ow, const int *__restrict__ first,
                                      const int *__restrict__ count, const int *__restrict__ coef, int ksize)
{
    const size_t total = (size_t)n * rows * ow;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        const int ox = (int)(i % ow);
        const size_t r = i / ow;
        const int y = (int)(r % rows) + y0, img = (int)(r / rows);
        const uint8_t *src = rgb + (((size_t)img * h + y) * w + first[ox]) * 3;
        const int *k = coef + (size_t)ox * ksize;
        int s0 = 1 << (PRE_BITS - 1), s1 = s0, s2 = s0;
        for (int x = 0; x < count[ox]; x++) {
            const int c = k[x];
            s0 += (int)src[3 * x] * c;
            s1 += (int)src[3 * x + 1] * c;
            s2 += (int)src[3 * x + 2] * c;
        }
        uint8_t *dst = tmp + i * 3;
        dst[0] = (uint8_t)clip8(s0);
        dst[1] = (uint8_t)clip8(s1);
        dst[2] = (uint8_t)clip8(s2);
    }
}

// Vertical pass and normalisation: out[n][c][oy][ox] = (q / 255 - mean[c]) /
// std[c], q the 8-bit resampled value.
__global__ void pre_vertical_kernel(const uint8_t *__restrict__ tmp, float *__restrict__ out, int n, int y0, int rows,
                                    int oh, int ow, const int *__restrict__ first, const int *__restrict__ count,
                                    const int *__restrict__ coef, int ksize, float m0, float m1, float m2, float d0,
                                    float d1, float d2)
{
    const size_t total = (size_t)n * oh * ow;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        const int ox = (int)(i % ow);
        const size_t r = i / ow;
        const int oy = (int)(r % oh), img = (int)(r / oh);
        const uint8_t *src = tmp + (((size_t)img * rows + (first[oy] - y0)) * ow + ox) * 3;
        const int *k = coef + (size_t)oy * ksize;
        int s0 = 1 << (PRE_BITS - 1), s1 = s0, s2 = s0;
        for (int y = 0; y < count[oy]; y++) {
            const int c = k[y];
            const uint8_t *p = src + (size_t)y * ow * 3;
            s0 += (int)p[0] * c;
            s1 += (int)p[1] * c;
            s2 += (int)p[2] * c;
        }
        const size_t plane = (size_t)oh * ow, o = (size_t)img * 3 * plane + (size_t)oy * ow + ox;
        out[o] = __fdiv_rn(__fsub_rn(__fdiv_rn((float)clip8(s0), 255.0f), m0), d0);
        out[o + plane] = __fdiv_rn(__fsub_rn(__fdiv_rn((float)clip8(s1), 255.0f), m1), d1);
        out[o + 2 * plane] = __fdiv_rn(__fsub_rn(__fdiv_rn((float)clip8(s2), 255.0f), m2), d2);
    }
}

}  // namespace

}  // namespace tcg

using namespace tcg;

extern "C" {

bool tcg_preprocess_rgb8(float *pixels, const uint8_t *rgb, int n, int height, int width, int image,
                         const float mean[3], const float std[3], int interpolation)
{
    if (!need_ctx()) return false;
    if (n < 0 || height <= 0 || width <= 0 || image <= 0) return fail("tcg_preprocess_rgb8: bad sizes");
    if (interpolation != 0 && interpolation != 1)
        return fail("tcg_preprocess_rgb8: interpolation %d is not bicubic (0) or bilinear (1)", interpolation);
    if (!mean || !std) return fail("tcg_preprocess_rgb8: null mean or std");
    for (int c = 0; c < 3; c++)
        if (!(std[c] != 0.0f)) return fail("tcg_preprocess_rgb8: std[%d] is zero", c);
    if (n == 0) return true;
    if (!pixels || !rgb) return fail("tcg_preprocess_rgb8: null pointer");
    // resize the shorter side to `image` (the longer one to the truncated
    // proportional length), then the centre crop, offsets rounded half to even
    const int shorter = height < width ? height : width, longer = height < width ? width : height;
    const int resized_long = (int)((double)image * (double)longer / (double)shorter);
    const int rh = width <= height ? resized_long : image;
    const int rw = width <= height ? image : resized_long;
    if (rh < image || rw < image) return fail("tcg_preprocess_rgb8: resized %dx%d smaller than the crop", rh, rw);
    const int top = (int)nearbyint((rh - image) / 2.0), left = (int)nearbyint((rw - image) / 2.0);
    const Axis hx = axis_coeffs(width, rw, interpolation, left, image);
    const Axis vy = axis_coeffs(height, rh, interpolation, top, image);
    // the input rows the vertical pass reads
    int y0 = height, y1 = 0;
    for (int i = 0; i < image; i++) {
        y0 = vy.first[i] < y0 ? vy.first[i] : y0;
        y1 = vy.first[i] + vy.count[i] > y1 ? vy.first[i] + vy.count[i] : y1;
    }
    const int rows = y1 - y0;
    // device copies of the tables and the 8-bit intermediate, in the scratch
    const size_t ints = (size_t)image * (2 + hx.ksize) + (size_t)image * (2 + vy.ksize);
    const size_t tmp_bytes = (size_t)n * rows * image * 3;
    const size_t table_bytes = (ints * sizeof(int) + 255) & ~(size_t)255;
    unsigned char *buf = (unsigned char *)scratch(table_bytes + tmp_bytes);
    if (!buf) return false;
    std::vector<int> host(ints);
    size_t at = 0;
    auto put = [&](const std::vector<int> &v) {
        const size_t start = at;
        memcpy(host.data() + at, v.data(), v.size() * sizeof(int));
        at += v.size();
        return start;
    };
    const size_t hf = put(hx.first), hc = put(hx.count), hk = put(hx.coef);
    const size_t vf = put(vy.first), vc = put(vy.count), vk = put(vy.coef);
    cudaStream_t s = ctx().cur;
    TCG_CUDA(cudaMemcpyAsync(buf, host.data(), ints * sizeof(int), cudaMemcpyHostToDevice, s));
    // the host table must outlive the copy
    TCG_CUDA(cudaStreamSynchronize(s));
    const int *d = (const int *)buf;
    uint8_t *tmp = buf + table_bytes;
    const size_t h_items = (size_t)n * rows * image, v_items = (size_t)n * image * image;
    const unsigned cap = (unsigned)(ctx().sms * 8);
    pre_horizontal_kernel<<<ceil_div(h_items, 256) < cap ? ceil_div(h_items, 256) : cap, 256, 0, s>>>(
        rgb, tmp, n, height, width, y0, rows, image, d + hf, d + hc, d + hk, hx.ksize);
    TCG_LAUNCHED();
    pre_vertical_kernel<<<ceil_div(v_items, 256) < cap ? ceil_div(v_items, 256) : cap, 256, 0, s>>>(
        tmp, pixels, n, y0, rows, image, image, d + vf, d + vc, d + vk, vy.ksize, mean[0], mean[1], mean[2], std[0],
        std[1], std[2]);
    TCG_LAUNCHED();
    return true;
}

bool tcg_vit_preprocess(const tc_vit_t *m, float *pixels, const uint8_t *rgb, int n, int height, int width)
{
    if (!m) return fail("tcg_vit_preprocess: null model");
    int interp = 0;                         // bicubic: open_clip's default when the key is absent
    gguf_str_t s;
    if (gguf_get_str(&m->gguf, "clip-vit.preprocess.interpolation", &s)) {
        if (gguf_str_eq(s, "bicubic")) interp = 0;
        else if (gguf_str_eq(s, "bilinear")) interp = 1;
        else {
            char b[64];
            gguf_str_cstr(b, sizeof b, s);
            return fail("tcg_vit_preprocess: interpolation '%s' not implemented (bicubic, bilinear)", b);
        }
    }
    if (gguf_get_str(&m->gguf, "clip-vit.preprocess.resize_mode", &s) && !gguf_str_eq(s, "shortest")) {
        char b[64];
        gguf_str_cstr(b, sizeof b, s);
        return fail("tcg_vit_preprocess: resize_mode '%s' not implemented (shortest)", b);
    }
    return tcg_preprocess_rgb8(pixels, rgb, n, height, width, m->image, m->mean, m->std, interp);
}

}  // extern "C"
