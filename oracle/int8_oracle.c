/* CPU INT8 convolution oracle (test infrastructure only: the checker for the
 * device INT8 convolution, never part of the product path).
 *
 * The reference (phucb2/yolo-baremetal) has no INT8 code, so parity here is
 * against this restatement of the INT8 scheme the benchmark specifies
 * (weights int8 symmetric per output channel, scale = max|w| / 127;
 * activations int8 per tensor; int32 accumulation; round-half-even
 * requantisation).  The fixed rules, shared with the library's host
 * quantiser (which computes them independently, in its own code):
 *
 *   s_w[c]  = m > 0 ? m / 127 : 1, m = max |w[c,...]|          (float)
 *   wq      = clamp(rint(w / s_w[c]), -127, 127)               (float, half-even)
 *   bq[c]   = clamp(llrint(b / (s_in * s_w[c])), +-(2^31 - 1)) (double)
 *   ratio   = s_in * s_w[c] / s_t, s_t = s_pre with a LUT, else s_out (double)
 *             = M * 2^-sh, M in [2^30, 2^31), from frexp;  sh > 62: M = 0, sh = 1
 *   y       = rshift_rne((acc + bq) * M, sh)   (64-bit, floor + half-even carry)
 *   out     = LUT ? lut[clamp(y, -128, 127) + 128] : clamp(y, -127, 127)
 *   lut[i]  = clamp(llrint(silu((i - 128) * s_pre) / s_out), -127, 127) (double)
 *
 * Tensors are NHWC int8; padding contributes zero.  */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>

static int64_t rshift_rne(int64_t p, int sh) {
    int64_t q = p >> sh; /* arithmetic: floor */
    const int64_t rem = p - (q << sh);
    const int64_t half = (int64_t)1 << (sh - 1);
    if (rem > half || (rem == half && (q & 1))) q += 1;
    return q;
}

static int clampi(int64_t v, int lo, int hi) { return v < lo ? lo : v > hi ? hi : (int)v; }

/* ratio -> (M, sh); returns 0 on success, -1 when the ratio is too large. */
int orc_i8_multiplier(double ratio, int32_t* mult, int32_t* shift) {
    if (!(ratio > 0.0)) {
        *mult = 0;
        *shift = 1;
        return 0;
    }
    int e = 0;
    const double f = frexp(ratio, &e); /* ratio = f * 2^e, f in [0.5, 1) */
    long long m = llrint(f * 2147483648.0);
    if (m == 2147483648LL) {
        m = 1073741824LL;
        e += 1;
    }
    const int sh = 31 - e;
    if (sh < 1) return -1;
    if (sh > 62) {
        *mult = 0;
        *shift = 1;
        return 0;
    }
    *mult = (int32_t)m;
    *shift = sh;
    return 0;
}

/* Quantises one convolution: w [co][ci][kh][kw] fp32, b [co] or NULL.
 * act_silu != 0 builds the SiLU table (pre-activation scale s_pre). */
int orc_i8_quantize_conv(const float* w, const float* b, int co, int ci, int kh, int kw, float s_in, float s_pre,
                         float s_out, int act_silu, int8_t* wq, int32_t* bq, int32_t* mult, int32_t* shift,
                         int8_t* lut) {
    const int per = ci * kh * kw;
    for (int c = 0; c < co; ++c) {
        float m = 0.0f;
        for (int i = 0; i < per; ++i) {
            const float a = fabsf(w[(size_t)c * per + i]);
            if (a > m) m = a;
        }
        const float sw = m > 0.0f ? m / 127.0f : 1.0f;
        for (int i = 0; i < per; ++i) {
            const float q = nearbyintf(w[(size_t)c * per + i] / sw);
            wq[(size_t)c * per + i] = (int8_t)(q < -127.0f ? -127 : q > 127.0f ? 127 : (int)q);
        }
        if (b) {
            const long long v = llrint((double)b[c] / ((double)s_in * (double)sw));
            bq[c] = (int32_t)(v < -2147483647LL ? -2147483647LL : v > 2147483647LL ? 2147483647LL : v);
        } else {
            bq[c] = 0;
        }
        const double st = act_silu ? (double)s_pre : (double)s_out;
        if (orc_i8_multiplier((double)s_in * (double)sw / st, &mult[c], &shift[c]) != 0) return -1;
    }
    if (act_silu) {
        for (int i = 0; i < 256; ++i) {
            const double x = (double)(i - 128) * (double)s_pre;
            const double y = x / (1.0 + exp(-x));
            const long long q = llrint(y / (double)s_out);
            lut[i] = (int8_t)(q < -127 ? -127 : q > 127 ? 127 : q);
        }
    }
    return 0;
}

/* y [B][Ho][Wo][co] = requant(conv(x [B][H][W][ci], wq) + bq). */
int orc_i8_conv(const int8_t* x, int B, int H, int W, int ci, const int8_t* wq, const int32_t* bq, const int32_t* mult,
                const int32_t* shift, const int8_t* lut, int co, int kh, int kw, int stride, int pad, int8_t* y) {
    const int Ho = (H + 2 * pad - kh) / stride + 1, Wo = (W + 2 * pad - kw) / stride + 1;
    if (Ho <= 0 || Wo <= 0) return -1;
#pragma omp parallel for collapse(2) schedule(dynamic)
    for (int b = 0; b < B; ++b)
        for (int oy = 0; oy < Ho; ++oy)
            for (int ox = 0; ox < Wo; ++ox)
                for (int c = 0; c < co; ++c) {
                    int64_t acc = bq[c];
                    for (int ky = 0; ky < kh; ++ky) {
                        const int iy = oy * stride - pad + ky;
                        if (iy < 0 || iy >= H) continue;
                        for (int kx = 0; kx < kw; ++kx) {
                            const int ix = ox * stride - pad + kx;
                            if (ix < 0 || ix >= W) continue;
                            const int8_t* xp = x + (((size_t)b * H + iy) * W + ix) * ci;
                            const int8_t* wp = wq + (size_t)c * ci * kh * kw + ky * kw + kx;
                            for (int i = 0; i < ci; ++i) acc += (int32_t)xp[i] * (int32_t)wp[(size_t)i * kh * kw];
                        }
                    }
                    const int64_t v = rshift_rne(acc * (int64_t)mult[c], shift[c]);
                    int8_t o;
                    if (lut) o = lut[clampi(v, -128, 127) + 128];
                    else o = (int8_t)clampi(v, -127, 127);
                    y[(((size_t)b * Ho + oy) * Wo + ox) * co + c] = o;
                }
    return 0;
}

int64_t orc_i8_rshift_rne(int64_t p, int sh) { return rshift_rne(p, sh); }
