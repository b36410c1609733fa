/* CPU restatement of the reference's image preprocessing and detection
 * lists -- TEST INFRASTRUCTURE ONLY (the checker of the device preprocess and
 * detection lists; nothing in the product links it).  Compiled with
 * -ffp-contract=off: every product and sum is rounded on its own, in the
 * reference's evaluation order.
 *
 *   orc_resize_align_corners  src/main.c:18-51 (resize_rgb_bilinear): source
 *       coordinate dx * (sw - 1) / (dw - 1), bilinear blend of the two rows'
 *       horizontal blends, rounded half up by (int)(v + 0.5f), clamped.
 *   orc_resize_half_pixel     tests/dump_model_stages.c:58-96
 *       (load_rgb_resized after decoding): source coordinate
 *       (x + 0.5) * iw / out_w - 0.5 truncated toward zero and clamped, the
 *       four-term weighted sum in the reference's order, truncated to uint8.
 *   orc_rgb_to_nchw           src/main.c:53-64 (preprocess): value / 255.0f,
 *       HWC RGB to planar NCHW.
 */
#include <math.h>
#include <stdint.h>

void orc_resize_align_corners(const uint8_t* src, int sw, int sh, uint8_t* dst, int dw, int dh) {
    if (sw <= 0 || sh <= 0 || dw <= 0 || dh <= 0) return;
    for (int dy = 0; dy < dh; dy++) {
        for (int dx = 0; dx < dw; dx++) {
            const float sx = (dw == 1) ? 0.f : (float)dx * (float)(sw - 1) / (float)(dw - 1);
            const float sy = (dh == 1) ? 0.f : (float)dy * (float)(sh - 1) / (float)(dh - 1);
            const int x0 = (int)floorf(sx), y0 = (int)floorf(sy);
            const int x1 = x0 + 1 < sw ? x0 + 1 : x0;
            const int y1 = y0 + 1 < sh ? y0 + 1 : y0;
            const float fx = sx - (float)x0, fy = sy - (float)y0;
            for (int c = 0; c < 3; c++) {
                const float a = (float)src[(y0 * sw + x0) * 3 + c];
                const float b = (float)src[(y0 * sw + x1) * 3 + c];
                const float d = (float)src[(y1 * sw + x0) * 3 + c];
                const float e = (float)src[(y1 * sw + x1) * 3 + c];
                const float top = a * (1.f - fx) + b * fx;
                const float bot = d * (1.f - fx) + e * fx;
                const float v = top * (1.f - fy) + bot * fy;
                int iv = (int)(v + 0.5f);
                iv = iv < 0 ? 0 : iv > 255 ? 255 : iv;
                dst[(dy * dw + dx) * 3 + c] = (uint8_t)iv;
            }
        }
    }
}

void orc_resize_half_pixel(const uint8_t* src, int iw, int ih, uint8_t* dst, int out_w, int out_h) {
    for (int y = 0; y < out_h; y++) {
        for (int x = 0; x < out_w; x++) {
            const float fx = (x + 0.5f) * (float)iw / (float)out_w - 0.5f;
            const float fy = (y + 0.5f) * (float)ih / (float)out_h - 0.5f;
            int sx = (int)fx, sy = (int)fy;
            sx = sx < 0 ? 0 : sx >= iw ? iw - 1 : sx;
            sy = sy < 0 ? 0 : sy >= ih ? ih - 1 : sy;
            const int sx1 = sx + 1 < iw ? sx + 1 : sx;
            const int sy1 = sy + 1 < ih ? sy + 1 : sy;
            const float tx = fx - (float)sx, ty = fy - (float)sy;
            for (int c = 0; c < 3; c++) {
                const float a = src[(sy * iw + sx) * 3 + c];
                const float b = src[(sy * iw + sx1) * 3 + c];
                const float d = src[(sy1 * iw + sx) * 3 + c];
                const float e = src[(sy1 * iw + sx1) * 3 + c];
                const float v = a * (1 - tx) * (1 - ty) + b * tx * (1 - ty) + d * (1 - tx) * ty + e * tx * ty;
                dst[(y * out_w + x) * 3 + c] = (uint8_t)(v < 0 ? 0 : (v > 255 ? 255 : v));
            }
        }
    }
}

void orc_rgb_to_nchw(const uint8_t* rgb, int w, int h, float* nchw) {
    const int plane = h * w;
    for (int i = 0; i < plane; i++)
        for (int c = 0; c < 3; c++) nchw[c * plane + i] = rgb[i * 3 + c] / 255.0f;
}

/* decode_detections (src/detection.c:3-34) for one image: rows [n][feat]
 * (x1, y1, x2, y2, score, class, ...); keeps the rows whose score is not
 * <= threshold, in row order, until `capacity` are kept.  out: per kept row
 * 5 floats and the class as int (the layout of detection_t).  Returns the
 * count. */
typedef struct {
    float x1, y1, x2, y2, score;
    int class_id;
} orc_det_t;

int orc_decode_detections(const float* rows, int n, int feat, float threshold, int capacity, orc_det_t* out) {
    int count = 0;
    for (int i = 0; i < n; i++) {
        const float* r = rows + (long)i * feat;
        if (r[4] <= threshold) continue;
        if (count >= capacity) break;
        orc_det_t* d = &out[count++];
        d->x1 = r[0];
        d->y1 = r[1];
        d->x2 = r[2];
        d->y2 = r[3];
        d->score = r[4];
        d->class_id = (int)r[5];
    }
    return count;
}
