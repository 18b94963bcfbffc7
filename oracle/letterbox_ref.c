/* CPU restatement of the reference letterbox preprocess, TEST INFRASTRUCTURE ONLY.
 *
 * Follows imageloader/src/preprocess.cpp:15-147 (preprocess_letterbox_direct):
 *   ratio    = min(W / src_w, H / src_h)                      float division (:27)
 *   scaled   = clamp(round(src * ratio), 1, target)           roundf, half away (:28-29)
 *   pad      = (target - scaled) / 2                          integer division (:31-32)
 *   inv      = 1.0f / ratio                                   (:54)
 *   per column dx: sx = dx * inv, x0 = (int)sx clamped to src_w - 2 when src_w > 1,
 *                  x1 = x0 + 1 < src_w ? x0 + 1 : x0, fx = sx - x0       (:59-66)
 *   per row dy:    the same for y; wy0 = (1 - fy) * scale, wy1 = fy * scale (:82-89)
 *   value = (p00*w0 + p10*w1)*wy0 + (p01*w0 + p11*w1)*wy1                  (:106-108)
 *   pad_value outside the scaled image; gray replicated to 3 planes, RGBA drops alpha.
 * The reference is compiled with -ffp-contract=fast, and its compiled value is the
 * contraction fma(fma(p00, w0, p10*w1), wy0, fma(p01, w0, p11*w1) * wy1): the
 * products and sums below are spelled out with fmaf in exactly that order, and this
 * file is compiled with -ffp-contract=off so that nothing else is fused. Pinned
 * bit-exact against the reference library built from its sources (golden fixtures in
 * tests/golden/letterbox_ref.npz).
 *
 * Output: out[3][H][W] float32 (NCHW planes R, G, B); meta[8] = target_w, target_h,
 * orig_w, orig_h, pad_x, pad_y, scaled_w, scaled_h; *ratio_out = ratio.
 * Returns 0, or -1 for an empty image, a channel count other than 1/3/4 or a target
 * below one pixel.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>

int letterbox_ref(const uint8_t* src, int src_h, int src_w, int ch, int W, int H, float scale, float pad,
                  float* out, int32_t* meta, float* ratio_out) {
    if (!src || src_h <= 0 || src_w <= 0 || W <= 0 || H <= 0 || (ch != 1 && ch != 3 && ch != 4)) return -1;
    const float ratio = fminf((float)W / (float)src_w, (float)H / (float)src_h);
    int sw = (int)roundf((float)src_w * ratio), sh = (int)roundf((float)src_h * ratio);
    sw = sw < 1 ? 1 : (sw > W ? W : sw);
    sh = sh < 1 ? 1 : (sh > H ? H : sh);
    const int px = (W - sw) / 2, py = (H - sh) / 2;
    const size_t plane = (size_t)W * H;
    for (size_t i = 0; i < 3 * plane; ++i) out[i] = pad;
    const float inv = 1.0f / ratio;
    for (int dy = 0; dy < sh; ++dy) {
        const float sy = (float)dy * inv;
        int y0 = (int)sy;
        if (y0 > src_h - 2 && src_h > 1) y0 = src_h - 2;
        const int y1 = y0 + 1 < src_h ? y0 + 1 : y0;
        const float fy = sy - (float)y0;
        const float wy0 = (1.0f - fy) * scale, wy1 = fy * scale;
        for (int dx = 0; dx < sw; ++dx) {
            const float sx = (float)dx * inv;
            int x0 = (int)sx;
            if (x0 > src_w - 2 && src_w > 1) x0 = src_w - 2;
            const int x1 = x0 + 1 < src_w ? x0 + 1 : x0;
            const float fx = sx - (float)x0;
            const float w0 = 1.0f - fx, w1 = fx;
            const size_t o = (size_t)(dy + py) * W + (size_t)(dx + px);
            for (int c = 0; c < 3; ++c) {
                const int cc = ch == 1 ? 0 : c;
                const float p00 = src[((size_t)y0 * src_w + x0) * ch + cc], p10 = src[((size_t)y0 * src_w + x1) * ch + cc];
                const float p01 = src[((size_t)y1 * src_w + x0) * ch + cc], p11 = src[((size_t)y1 * src_w + x1) * ch + cc];
                const float top = fmaf(p00, w0, p10 * w1);
                const float bot = fmaf(p01, w0, p11 * w1);
                out[c * plane + o] = fmaf(top, wy0, bot * wy1);
            }
        }
    }
    meta[0] = W; meta[1] = H; meta[2] = src_w; meta[3] = src_h;
    meta[4] = px; meta[5] = py; meta[6] = sw; meta[7] = sh;
    *ratio_out = ratio;
    return 0;
}
