/*
 * ORACLE (test infrastructure only) -- CPU restatement of the reference's image
 * preprocessing, csrc/cpu/preprocessing.cpp (Aedelon/mast3r-runtime), the path every
 * native engine takes for an image whose size differs from the model's.
 *
 * Only tests/ may load this library, and only as the checker.
 *
 *   resize + centre crop   preprocessing.cpp:29-63: scale = max(dst_h / src_h,
 *                          dst_w / src_w) in float, new = (int)(src * scale), bilinear
 *                          resize to new_h x new_w, crop [start, start + dst) with
 *                          start = (new - dst) / 2.  The reference takes a square
 *                          target (dst_h == dst_w); a rectangular one follows the same
 *                          formulas.  Where truncation makes new < dst the reference
 *                          reads past its resized buffer; here (and on the GPU) such
 *                          rows / columns are clamped to the last one.
 *   bilinear resize        preprocessing.cpp:84-129: scale = src / dst (float),
 *                          s = d * scale, i0 = (int)s, i1 = min(i0 + 1, src - 1),
 *                          weights (1-fx)(1-fy), fx(1-fy), (1-fx)fy, fx fy, the sum
 *                          w00 v00 + w01 v01 + w10 v10 + w11 v11 left to right, every
 *                          multiply and add rounded separately (no FMA), clamped to
 *                          [0, 255] and truncated to uint8.
 *   normalise              preprocessing.cpp:65-82: (v / 255 - mean) / std, HWC -> CHW
 *
 * Build: oracle/Makefile (-ffp-contract=off).
 */
#include <stdint.h>

static int imin(int a, int b) { return a < b ? a : b; }

void oracle_resize_crop(const uint8_t* src, int src_h, int src_w, uint8_t* dst, int dst_h, int dst_w) {
    const float sc_h = (float)dst_h / (float)src_h;
    const float sc_w = (float)dst_w / (float)src_w;
    const float scale = sc_h > sc_w ? sc_h : sc_w;
    const int new_h = (int)((float)src_h * scale);
    const int new_w = (int)((float)src_w * scale);
    const int start_h = (new_h - dst_h) / 2;
    const int start_w = (new_w - dst_w) / 2;
    const float scale_y = (float)src_h / (float)new_h;
    const float scale_x = (float)src_w / (float)new_w;
    for (int y = 0; y < dst_h; ++y) {
        const int ry = imin(start_h + y, new_h - 1);
        const float sy = (float)ry * scale_y;
        const int y0 = (int)sy;
        const int y1 = imin(y0 + 1, src_h - 1);
        const float fy = sy - (float)y0;
        for (int x = 0; x < dst_w; ++x) {
            const int rx = imin(start_w + x, new_w - 1);
            const float sx = (float)rx * scale_x;
            const int x0 = (int)sx;
            const int x1 = imin(x0 + 1, src_w - 1);
            const float fx = sx - (float)x0;
            const float w00 = (1.0f - fx) * (1.0f - fy);
            const float w01 = fx * (1.0f - fy);
            const float w10 = (1.0f - fx) * fy;
            const float w11 = fx * fy;
            for (int c = 0; c < 3; ++c) {
                const float v00 = (float)src[((long)y0 * src_w + x0) * 3 + c];
                const float v01 = (float)src[((long)y0 * src_w + x1) * 3 + c];
                const float v10 = (float)src[((long)y1 * src_w + x0) * 3 + c];
                const float v11 = (float)src[((long)y1 * src_w + x1) * 3 + c];
                float val = w00 * v00;
                val = val + w01 * v01;
                val = val + w10 * v10;
                val = val + w11 * v11;
                val = val < 0.0f ? 0.0f : (val > 255.0f ? 255.0f : val);
                dst[((long)y * dst_w + x) * 3 + c] = (uint8_t)val;
            }
        }
    }
}

void oracle_normalize_chw(const uint8_t* img, int h, int w, float* out) {
    static const float mean[3] = {0.485f, 0.456f, 0.406f};
    static const float stdv[3] = {0.229f, 0.224f, 0.225f};
    const long size = (long)h * w;
    for (long i = 0; i < size; ++i)
        for (int c = 0; c < 3; ++c) {
            const float v = (float)img[i * 3 + c] / 255.0f;
            out[c * size + i] = (v - mean[c]) / stdv[c];
        }
}
