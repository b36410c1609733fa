#ifndef YB_INT8_H
#define YB_INT8_H

/* INT8 convolution on the B200 tensor cores (tcgen05.mma kind::i8, int32
 * accumulation in tensor memory) with the requantisation fused into the
 * epilogue.  No counterpart in the reference: phucb2/yolo-baremetal has no
 * INT8 path; these entry points implement the INT8 scheme its benchmark
 * specifies (weights int8 symmetric per output channel with scale
 * max|w| / 127, activations int8 per tensor, int32 accumulation,
 * round-half-even requantisation), for one convolution layer.
 *
 * Quantisation rules (yb_int8_quantize_conv):
 *   s_w[c] = m > 0 ? m / 127 : 1 with m = max |w[c,...]|        (float)
 *   wq     = clamp(rint(w / s_w[c]), -127, 127)                 (float, half-even)
 *   bq[c]  = rint(b[c] / (s_in * s_w[c])), clamped to int32     (double)
 *   s_in * s_w[c] / s_t = mult[c] * 2^-shift[c], mult in [2^30, 2^31),
 *            s_t = s_pre when act_silu, else s_out             (double, frexp)
 *   lut[i] = clamp(rint(silu((i - 128) * s_pre) / s_out), -127, 127)
 * Layer arithmetic (yb_int8_conv_run), per output element:
 *   acc = bq[c] + sum x * wq                                    (exact)
 *   y   = ((acc * mult[c]) >> shift[c]) rounded half to even    (64-bit)
 *   out = lut ? lut[clamp(y, -128, 127) + 128] : clamp(y, -127, 127)
 * Activations are NHWC int8; zero padding. */

#include <stdint.h>

#include "status.h"

#ifdef __cplusplus
extern "C" {
#endif

/* w [co][ci][kh][kw] fp32, b [co] or NULL.  Outputs: wq [co][ci][kh][kw],
 * bq, mult, shift [co]; lut [256] when act_silu (else untouched, may be
 * NULL).  ERROR_INVALID_DIMS when a ratio s_in*s_w/s_t is 2^30 or more. */
status_t yb_int8_quantize_conv(const float* w, const float* b, int co, int ci, int kh, int kw, float s_in,
                               float s_pre, float s_out, int act_silu, int8_t* wq, int32_t* bq, int32_t* mult,
                               int32_t* shift, int8_t* lut);

/* Packs and uploads one quantised convolution to `device` (host inputs as
 * produced above; lut NULL for no activation).  co a multiple of 16 (<= 1024),
 * kh = kw in {1, 3}.  *conv receives an opaque handle. */
status_t yb_int8_conv_create(int device, const int8_t* wq, const int32_t* bq, const int32_t* mult,
                             const int32_t* shift, const int8_t* lut, int co, int ci, int kh, int kw, int stride,
                             int pad, void** conv);

/* Channel stride the input must have: ci rounded up to a multiple of 32
 * (the extra channels must be zero). */
int yb_int8_conv_ci_pad(void* conv);

/* d_x: device NHWC int8 [B,H,W,ci_pad]; d_y: device NHWC int8
 * [B,Ho,Wo,co].  Enqueued on `stream` (NULL = the default stream); does not
 * synchronize.  A device timeout inside the kernel is reported by the next
 * call or by yb_int8_conv_destroy as ERROR_DEVICE. */
status_t yb_int8_conv_run(void* conv, const int8_t* d_x, int B, int H, int W, int8_t* d_y, void* stream);

/* Reads and clears the handle's device error word (synchronizes). */
status_t yb_int8_conv_check(void* conv);

status_t yb_int8_conv_destroy(void* conv);

#ifdef __cplusplus
}
#endif

#endif
