/* CPU INT8 YOLO26 forward -- TEST INFRASTRUCTURE ONLY (the checker of the
 * device INT8 path; nothing in the product links it).
 *
 * The reference has no INT8 code; this restates the INT8 scheme of the
 * benchmark (int8 symmetric per-output-channel weights, per-tensor int8
 * activations, int32 accumulation, round-half-even requantisation) over the
 * same graph as the FP32 oracle (yolo_oracle.c, which follows src/model.c,
 * src/layers.c and src/detect.c).  Every rule below is integer once the
 * per-tensor scales are fixed, so the device path must match it bit for bit
 * given the same scale table.
 *
 * Scale table: one float per named tensor.  A conv named P (its weight
 * prefix) writes tensor "P" (after its residual, if any) and, with SiLU, has
 * a pre-activation scale "P:pre".  Also "input", "<psa>.attn.ope" (attention
 * output plus positional term), and the dwconvs of the Detect head.
 *
 * Rules (see also int8_oracle.c for the per-layer arithmetic):
 *  - input: q = clamp(rint(x / s_input), -127, 127) in float.
 *  - Every tensor carries one scale per channel (concats keep their parts'
 *    scales).  A conv folds them into its weights: s_ref = scale of input
 *    channel 0, w_eff = (float)(w * s_c / s_ref) in double, then per output
 *    channel s_w = max|w_eff| / 127, wq = clamp(rint(w_eff / s_w)),
 *    bq = rint(b / (s_ref * s_w)); requant ratio s_ref * s_w / s_t as
 *    (M, sh) from frexp; y = rshift_rne(acc * M, sh).
 *  - SiLU: p = clamp(y, -128, 127), out = lut[p + 128], lut built in double
 *    from s_pre to the output scale.  No activation: clamp(y, -127, 127).
 *  - Residual r (scale s_r): out = clamp(v + rshift_rne(r * M_r, sh_r)),
 *    v the LUT value (SiLU) or the unclamped y (no activation);
 *    s_r / s_out = M_r * 2^-sh_r.
 *  - Max pool: int8 max, padding excluded.  Upsample and concat copy.
 *  - Depthwise 3x3: per-channel weight scales, same requantisation.
 *  - Attention (per head, kd = hd / 2): S = q.k (int32); t = min(255,
 *    rshift_rne((max_j S - S) * M_t, sh_t)) with s_qkv^2 / sqrt(kd) * 16 =
 *    M_t * 2^-sh_t; p = E[t], E[t] = rint(4096 exp(-t / 16)); l = sum p,
 *    o = sum p v (int64); a = div_rne(rshift_rne(o * M_o, sh_o), l) with
 *    s_qkv / s_ope = M_o * 2^-sh_o; plus the depthwise positional term of v
 *    requantised to s_ope; clamp(a + pe, -127, 127).
 *  - Detect's last 1x1 convs: float (acc) * (float)(s_ref * s_w[c]).
 */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

const float* orc_tensor_ptr(void* h, const char* name, int* dims4);
int orc_nc(void* h);
int orc_postprocess(const float* pred, int N, int nc, int max_det, int cap, float* out);
int orc_i8_multiplier(double ratio, int32_t* mult, int32_t* shift);

typedef struct {
    int8_t* d;
    float* cs; /* per-channel scales */
    int c, h, w;
    int own;
} q8;

typedef struct {
    void* m;
    const char* const* names;
    const float* scales;
    int n;
} i8ctx;

typedef void (*i8_stage_cb)(void* user, const char* name, const int8_t* data, const float* scales, int c, int h,
                            int w);

enum { I8_OK = 0, I8_ERR_MISSING = 5, I8_ERR_DIMS = 2, I8_ERR_SCALE = 6 };

static q8 q8_new(int c, int h, int w) {
    q8 f = {(int8_t*)calloc((size_t)c * h * w, 1), (float*)calloc((size_t)c, sizeof(float)), c, h, w, 1};
    return f;
}
static void q8_free(q8* f) {
    if (f->own) {
        free(f->d);
        free(f->cs);
    }
    f->d = NULL;
    f->cs = NULL;
}
static q8 q8_view(const q8* f, int c0, int c) {
    q8 v = {f->d + (size_t)c0 * f->h * f->w, f->cs + c0, c, f->h, f->w, 0};
    return v;
}
static void q8_set_scale(q8* f, float s) {
    for (int c = 0; c < f->c; ++c) f->cs[c] = s;
}

static int64_t rne(int64_t p, int sh) {
    int64_t q = p >> sh;
    const int64_t rem = p - (q << sh);
    const int64_t half = (int64_t)1 << (sh - 1);
    if (rem > half || (rem == half && (q & 1))) q += 1;
    return q;
}
static int64_t div_rne(int64_t a, int64_t l) {
    int64_t q = a / l, r = a % l;
    if (r < 0) {
        q -= 1;
        r += l;
    }
    if (2 * r > l || (2 * r == l && (q & 1))) q += 1;
    return q;
}
static int clampi(int64_t v, int lo, int hi) { return v < lo ? lo : v > hi ? hi : (int)v; }

static float scale_of(const i8ctx* x, const char* name) {
    for (int i = 0; i < x->n; ++i)
        if (strcmp(x->names[i], name) == 0) return x->scales[i];
    return -1.0f;
}

static int mult_of(double ratio, int32_t* m, int32_t* sh) { return orc_i8_multiplier(ratio, m, sh); }

typedef struct {
    int co, ci, kh, kw;
    int8_t* wq;
    int32_t *bq, *mult, *shift;
    float* deq;
    float s_ref;
} qconv_t;

static void qconv_free(qconv_t* q) {
    free(q->wq);
    free(q->bq);
    free(q->mult);
    free(q->shift);
    free(q->deq);
}

/* Quantises weights w [co][ci][kh][kw] (groups = 1) for an input with
 * per-channel scales cs; targets s_t (0: dequantised output). */
static int quantize(qconv_t* q, const float* w, const float* b, int co, int ci, int kh, int kw, const float* cs,
                    double s_t) {
    const int per = ci * kh * kw;
    q->co = co;
    q->ci = ci;
    q->kh = kh;
    q->kw = kw;
    q->s_ref = cs[0];
    q->wq = (int8_t*)malloc((size_t)co * per);
    q->bq = (int32_t*)malloc((size_t)co * 4);
    q->mult = (int32_t*)malloc((size_t)co * 4);
    q->shift = (int32_t*)malloc((size_t)co * 4);
    q->deq = (float*)malloc((size_t)co * 4);
    float* we = (float*)malloc((size_t)per * sizeof(float));
    int st = I8_OK;
    for (int o = 0; o < co && st == I8_OK; ++o) {
        float m = 0.0f;
        for (int i = 0; i < ci; ++i)
            for (int k = 0; k < kh * kw; ++k) {
                const int idx = i * kh * kw + k;
                we[idx] = (float)((double)w[(size_t)o * per + idx] * (double)cs[i] / (double)q->s_ref);
                if (fabsf(we[idx]) > m) m = fabsf(we[idx]);
            }
        const float sw = m > 0.0f ? m / 127.0f : 1.0f;
        for (int idx = 0; idx < per; ++idx) {
            const float v = nearbyintf(we[idx] / sw);
            q->wq[(size_t)o * per + idx] = (int8_t)(v < -127.0f ? -127 : v > 127.0f ? 127 : (int)v);
        }
        long long bv = b ? llrint((double)b[o] / ((double)q->s_ref * (double)sw)) : 0;
        bv = bv < -2147483647LL ? -2147483647LL : bv > 2147483647LL ? 2147483647LL : bv;
        q->bq[o] = (int32_t)bv;
        q->deq[o] = (float)((double)q->s_ref * (double)sw);
        if (s_t > 0.0) {
            if (mult_of((double)q->s_ref * (double)sw / s_t, &q->mult[o], &q->shift[o]) != 0) st = I8_ERR_SCALE;
        } else {
            q->mult[o] = 0;
            q->shift[o] = 1;
        }
    }
    free(we);
    return st;
}

static void build_lut(int8_t* lut, double s_pre, double s_out) {
    for (int i = 0; i < 256; ++i) {
        const double x = (double)(i - 128) * s_pre;
        const double y = x / (1.0 + exp(-x));
        const long long q = llrint(y / s_out);
        lut[i] = (int8_t)(q < -127 ? -127 : q > 127 ? 127 : q);
    }
}

/* Accumulator (bias included) of output channel o at (oy, ox). */
static int64_t acc_at(const qconv_t* q, const q8* in, int o, int oy, int ox, int stride, int pad) {
    int64_t acc = q->bq[o];
    for (int i = 0; i < q->ci; ++i)
        for (int ky = 0; ky < q->kh; ++ky) {
            const int iy = oy * stride - pad + ky;
            if (iy < 0 || iy >= in->h) continue;
            for (int kx = 0; kx < q->kw; ++kx) {
                const int ix = ox * stride - pad + kx;
                if (ix < 0 || ix >= in->w) continue;
                acc += (int32_t)in->d[((size_t)i * in->h + iy) * in->w + ix] *
                       (int32_t)q->wq[(((size_t)o * q->ci + i) * q->kh + ky) * q->kw + kx];
            }
        }
    return acc;
}

/* Conv named P (weights P.conv.weight / P.conv.bias): act SiLU when act,
 * residual res (single scale) when non-NULL; out gets scale table[P]. */
static int qconv(const i8ctx* x, const char* P, q8* out, const q8* in, int stride, int pad, int act, const q8* res) {
    char nm[160];
    int dims[4];
    snprintf(nm, sizeof nm, "%s.conv.weight", P);
    const float* w = orc_tensor_ptr(x->m, nm, dims);
    snprintf(nm, sizeof nm, "%s.conv.bias", P);
    const float* b = orc_tensor_ptr(x->m, nm, NULL);
    if (!w) return I8_ERR_MISSING;
    if (dims[1] != in->c || dims[0] != out->c) return I8_ERR_DIMS;
    const float s_out = scale_of(x, P);
    snprintf(nm, sizeof nm, "%s:pre", P);
    const float s_pre = act ? scale_of(x, nm) : 1.0f;
    if (!(s_out > 0.0f) || !(s_pre > 0.0f)) return I8_ERR_SCALE;
    qconv_t q;
    int st = quantize(&q, w, b, dims[0], dims[1], dims[2], dims[3], in->cs, act ? (double)s_pre : (double)s_out);
    int8_t lut[256];
    if (act) build_lut(lut, s_pre, s_out);
    int32_t mr = 0, shr = 1;
    if (st == I8_OK && res && mult_of((double)res->cs[0] / (double)s_out, &mr, &shr) != 0) st = I8_ERR_SCALE;
    /* Output channels in parallel: integer arithmetic, so the result does
     * not depend on the thread count. */
    if (st == I8_OK)
#pragma omp parallel for schedule(dynamic)
        for (int o = 0; o < out->c; ++o)
        for (int oy = 0; oy < out->h; ++oy)
            for (int ox = 0; ox < out->w; ++ox) {
                const int64_t y = rne(acc_at(&q, in, o, oy, ox, stride, pad) * q.mult[o], q.shift[o]);
                int64_t v = act ? (int64_t)lut[clampi(y, -128, 127) + 128] : y;
                const size_t oi = ((size_t)o * out->h + oy) * out->w + ox;
                if (res) v += rne((int64_t)res->d[oi] * mr, shr);
                out->d[oi] = (int8_t)clampi(v, -127, 127);
            }
    q8_set_scale(out, s_out);
    qconv_free(&q);
    return st;
}

/* Plain conv (weights P.weight / P.bias), dequantised to float [co][h*w]. */
static int qconv_deq(const i8ctx* x, const char* P, float* out, const q8* in) {
    char nm[160];
    int dims[4];
    snprintf(nm, sizeof nm, "%s.weight", P);
    const float* w = orc_tensor_ptr(x->m, nm, dims);
    snprintf(nm, sizeof nm, "%s.bias", P);
    const float* b = orc_tensor_ptr(x->m, nm, NULL);
    if (!w) return I8_ERR_MISSING;
    if (dims[1] != in->c) return I8_ERR_DIMS;
    qconv_t q;
    int st = quantize(&q, w, b, dims[0], dims[1], dims[2], dims[3], in->cs, 0.0);
    const int pad = (dims[2] - 1) / 2;
    if (st == I8_OK)
#pragma omp parallel for schedule(dynamic)
        for (int o = 0; o < q.co; ++o)
        for (int oy = 0; oy < in->h; ++oy)
            for (int ox = 0; ox < in->w; ++ox)
                out[((size_t)o * in->h + oy) * in->w + ox] = (float)acc_at(&q, in, o, oy, ox, 1, pad) * q.deq[o];
    qconv_free(&q);
    return st;
}

/* Depthwise 3x3 named P (P.conv.weight [C][1][3][3]) with SiLU. */
static int qdw(const i8ctx* x, const char* P, q8* out, const q8* in) {
    char nm[160];
    int dims[4];
    snprintf(nm, sizeof nm, "%s.conv.weight", P);
    const float* w = orc_tensor_ptr(x->m, nm, dims);
    snprintf(nm, sizeof nm, "%s.conv.bias", P);
    const float* b = orc_tensor_ptr(x->m, nm, NULL);
    if (!w) return I8_ERR_MISSING;
    const int C = in->c;
    if (dims[0] != C || dims[2] != 3) return I8_ERR_DIMS;
    const float s_out = scale_of(x, P);
    snprintf(nm, sizeof nm, "%s:pre", P);
    const float s_pre = scale_of(x, nm);
    if (!(s_out > 0.0f) || !(s_pre > 0.0f)) return I8_ERR_SCALE;
    int8_t lut[256];
    build_lut(lut, s_pre, s_out);
    int st = I8_OK;
#pragma omp parallel for schedule(dynamic) reduction(max : st)
    for (int c = 0; c < C; ++c) {
        qconv_t q;
        const float sc = in->cs[c];
        const int sq = quantize(&q, w + (size_t)c * 9, b ? b + c : NULL, 1, 1, 3, 3, &sc, (double)s_pre);
        if (sq > st) st = sq;
        q8 ch = q8_view(in, c, 1);
        for (int oy = 0; oy < in->h && sq == I8_OK; ++oy)
            for (int ox = 0; ox < in->w; ++ox) {
                const int64_t y = rne(acc_at(&q, &ch, 0, oy, ox, 1, 1) * q.mult[0], q.shift[0]);
                out->d[((size_t)c * in->h + oy) * in->w + ox] = lut[clampi(y, -128, 127) + 128];
            }
        qconv_free(&q);
    }
    q8_set_scale(out, s_out);
    return st;
}

static void qmaxpool(q8* out, const q8* in, int k) {
    const int pad = k / 2;
    for (int c = 0; c < in->c; ++c) {
        for (int y = 0; y < in->h; ++y)
            for (int xx = 0; xx < in->w; ++xx) {
                int m = -128;
                for (int ky = 0; ky < k; ++ky) {
                    const int iy = y - pad + ky;
                    if (iy < 0 || iy >= in->h) continue;
                    for (int kx = 0; kx < k; ++kx) {
                        const int ix = xx - pad + kx;
                        if (ix < 0 || ix >= in->w) continue;
                        const int v = in->d[((size_t)c * in->h + iy) * in->w + ix];
                        if (v > m) m = v;
                    }
                }
                out->d[((size_t)c * in->h + y) * in->w + xx] = (int8_t)m;
            }
        out->cs[c] = in->cs[c];
    }
}

static void q8_copy(q8* dst, const q8* src) {
    memcpy(dst->d, src->d, (size_t)src->c * src->h * src->w);
    memcpy(dst->cs, src->cs, (size_t)src->c * sizeof(float));
}

static int qbottleneck(const i8ctx* x, const char* p, q8* out, const q8* in, int shortcut) {
    char n1[200], n2[200], nm[200];
    snprintf(n1, sizeof n1, "%s.cv1", p);
    snprintf(n2, sizeof n2, "%s.cv2", p);
    int d1[4], d2[4];
    snprintf(nm, sizeof nm, "%s.conv.weight", n1);
    if (!orc_tensor_ptr(x->m, nm, d1)) return I8_ERR_MISSING;
    snprintf(nm, sizeof nm, "%s.conv.weight", n2);
    if (!orc_tensor_ptr(x->m, nm, d2)) return I8_ERR_MISSING;
    q8 t = q8_new(d1[0], in->h, in->w);
    int st = qconv(x, n1, &t, in, 1, (d1[2] - 1) / 2, 1, NULL);
    if (st == I8_OK) st = qconv(x, n2, out, &t, 1, (d2[2] - 1) / 2, 1, shortcut ? in : NULL);
    q8_free(&t);
    return st;
}

static int wdim0(const i8ctx* x, const char* fmt, const char* L) {
    char nm[200];
    int d[4];
    snprintf(nm, sizeof nm, fmt, L);
    return orc_tensor_ptr(x->m, nm, d) ? d[0] : 0;
}

static int qc3k2_plain(const i8ctx* x, const char* L, int n, int shortcut, q8* out, const q8* in) {
    char nm[220];
    const int ct = wdim0(x, "%s.cv1.conv.weight", L), ch = ct / 2;
    if (!ct) return I8_ERR_MISSING;
    q8 cat = q8_new((2 + n) * ch, in->h, in->w);
    q8 a = q8_view(&cat, 0, ct);
    snprintf(nm, sizeof nm, "%s.cv1", L);
    int st = qconv(x, nm, &a, in, 1, 0, 1, NULL);
    for (int i = 0; i < n && st == I8_OK; ++i) {
        q8 prev = q8_view(&cat, i == 0 ? ch : (1 + i) * ch, ch);
        q8 y = q8_view(&cat, (2 + i) * ch, ch);
        snprintf(nm, sizeof nm, "%s.m.%d", L, i);
        st = qbottleneck(x, nm, &y, &prev, shortcut);
    }
    snprintf(nm, sizeof nm, "%s.cv2", L);
    if (st == I8_OK) st = qconv(x, nm, out, &cat, 1, 0, 1, NULL);
    q8_free(&cat);
    return st;
}

static int qc3(const i8ctx* x, const char* P, int shortcut, q8* out, const q8* in) {
    char nm[220];
    const int cm = wdim0(x, "%s.cv1.conv.weight", P), c2 = wdim0(x, "%s.cv2.conv.weight", P);
    if (!cm || !c2) return I8_ERR_MISSING;
    q8 cat = q8_new(cm + c2, in->h, in->w);
    q8 y = q8_new(cm, in->h, in->w), z = q8_new(cm, in->h, in->w);
    q8 v2 = q8_view(&cat, cm, c2);
    snprintf(nm, sizeof nm, "%s.cv1", P);
    int st = qconv(x, nm, &y, in, 1, 0, 1, NULL);
    snprintf(nm, sizeof nm, "%s.cv2", P);
    if (st == I8_OK) st = qconv(x, nm, &v2, in, 1, 0, 1, NULL);
    q8 *cur = &y, *nxt = &z;
    for (int i = 0; st == I8_OK; ++i) {
        snprintf(nm, sizeof nm, "%s.m.%d", P, i);
        char probe[240];
        int d[4];
        snprintf(probe, sizeof probe, "%s.cv1.conv.weight", nm);
        if (!orc_tensor_ptr(x->m, probe, d)) break;
        st = qbottleneck(x, nm, nxt, cur, shortcut);
        q8* t = cur;
        cur = nxt;
        nxt = t;
    }
    q8 head = q8_view(&cat, 0, cm);
    q8_copy(&head, cur);
    snprintf(nm, sizeof nm, "%s.cv3", P);
    if (st == I8_OK) st = qconv(x, nm, out, &cat, 1, 0, 1, NULL);
    q8_free(&y);
    q8_free(&z);
    q8_free(&cat);
    return st;
}

static int qc3k2_c3k(const i8ctx* x, const char* L, q8* out, const q8* in) {
    char nm[220];
    const int ch = wdim0(x, "%s.cv1.conv.weight", L) / 2;
    char k3n[220];
    snprintf(k3n, sizeof k3n, "%s.m.0", L);
    const int c3o = wdim0(x, "%s.cv3.conv.weight", k3n);
    if (!ch || !c3o) return I8_ERR_MISSING;
    int n = 0;
    for (;; ++n) {
        char pn[220];
        snprintf(pn, sizeof pn, "%s.m.%d", L, n);
        if (!wdim0(x, "%s.cv3.conv.weight", pn)) break;
    }
    q8 cat = q8_new(2 * ch + n * c3o, in->h, in->w);
    q8 a = q8_view(&cat, 0, 2 * ch);
    snprintf(nm, sizeof nm, "%s.cv1", L);
    int st = qconv(x, nm, &a, in, 1, 0, 1, NULL);
    for (int i = 0; i < n && st == I8_OK; ++i) {
        q8 b = q8_view(&cat, i == 0 ? ch : 2 * ch + (i - 1) * c3o, i == 0 ? ch : c3o);
        q8 o = q8_view(&cat, 2 * ch + i * c3o, c3o);
        snprintf(nm, sizeof nm, "%s.m.%d", L, i);
        st = qc3(x, nm, 1, &o, &b);
    }
    snprintf(nm, sizeof nm, "%s.cv2", L);
    if (st == I8_OK) st = qconv(x, nm, out, &cat, 1, 0, 1, NULL);
    q8_free(&cat);
    return st;
}

static int qsppf(const i8ctx* x, const char* L, int k, int n_pool, int shortcut, q8* out, const q8* in) {
    char nm[220];
    const int c = wdim0(x, "%s.cv1.conv.weight", L);
    if (!c) return I8_ERR_MISSING;
    q8 cat = q8_new(c * (n_pool + 1), in->h, in->w);
    q8 s0 = q8_view(&cat, 0, c);
    snprintf(nm, sizeof nm, "%s.cv1", L);
    int st = qconv(x, nm, &s0, in, 1, 0, 0, NULL);
    for (int j = 0; j < n_pool && st == I8_OK; ++j) {
        q8 a = q8_view(&cat, j * c, c), b = q8_view(&cat, (j + 1) * c, c);
        qmaxpool(&b, &a, k);
    }
    snprintf(nm, sizeof nm, "%s.cv2", L);
    if (st == I8_OK) st = qconv(x, nm, out, &cat, 1, 0, 1, (shortcut && in->c == out->c) ? in : NULL);
    q8_free(&cat);
    return st;
}

/* Attention of PSA block P on x (layers.c:310-405) with the integer softmax:
 * ope (attention output + positional term) at scale table[P.attn.ope]. */
static int qattention(const i8ctx* x, const char* P, int heads, q8* ope, const q8* in) {
    char nm[220];
    const int dim = in->c, N = in->h * in->w;
    if (dim % heads) return I8_ERR_DIMS;
    const int hd = dim / heads, kd = (int)((float)hd * 0.5f);
    snprintf(nm, sizeof nm, "%s.attn.qkv", P);
    const int cq = wdim0(x, "%s.conv.weight", nm);
    if (cq != dim + 2 * kd * heads) return I8_ERR_DIMS;
    q8 qkv = q8_new(cq, in->h, in->w);
    int st = qconv(x, nm, &qkv, in, 1, 0, 0, NULL);
    const double s_qkv = qkv.cs[0];
    snprintf(nm, sizeof nm, "%s.attn.ope", P);
    const float s_ope = scale_of(x, nm);
    if (!(s_ope > 0.0f)) st = I8_ERR_SCALE;
    int32_t mt = 0, sht = 1, mo = 0, sho = 1;
    if (st == I8_OK && (mult_of(s_qkv * s_qkv / sqrt((double)kd) * 16.0, &mt, &sht) != 0 ||
                        mult_of(s_qkv / (double)s_ope, &mo, &sho) != 0))
        st = I8_ERR_SCALE;
    int32_t E[256];
    for (int t = 0; t < 256; ++t) E[t] = (int32_t)llrint(4096.0 * exp(-(double)t / 16.0));
    /* Positional term: depthwise 3x3 of v (all heads), requantised to s_ope. */
    int dims[4];
    snprintf(nm, sizeof nm, "%s.attn.pe.conv.weight", P);
    const float* pw = orc_tensor_ptr(x->m, nm, dims);
    snprintf(nm, sizeof nm, "%s.attn.pe.conv.bias", P);
    const float* pb = orc_tensor_ptr(x->m, nm, NULL);
    if (!pw || dims[0] != dim) st = st == I8_OK ? I8_ERR_MISSING : st;
    /* Per-channel quantised positional weights (input scale s_qkv). */
    qconv_t* pq = (qconv_t*)calloc((size_t)dim, sizeof(qconv_t));
    const float sv = (float)s_qkv;
    for (int ch = 0; ch < dim && st == I8_OK && pw; ++ch)
        st = quantize(&pq[ch], pw + (size_t)ch * 9, pb ? pb + ch : NULL, 1, 1, 3, 3, &sv, (double)s_ope);
    const int blk = 2 * kd + hd;
    for (int h = 0; h < heads && st == I8_OK; ++h) {
        const int8_t* q = qkv.d + (size_t)(h * blk) * N;
        const int8_t* k = qkv.d + (size_t)(h * blk + kd) * N;
        const int8_t* v = qkv.d + (size_t)(h * blk + 2 * kd) * N;
        /* Query rows in parallel, each with its own score row and sums. */
#pragma omp parallel
        {
        int64_t* o = (int64_t*)malloc((size_t)hd * sizeof(int64_t));
        int32_t* S = (int32_t*)malloc((size_t)N * sizeof(int32_t));
#pragma omp for schedule(static)
        for (int i = 0; i < N; ++i) {
            int32_t mx = INT32_MIN;
            for (int j = 0; j < N; ++j) {
                int32_t s = 0;
                for (int d = 0; d < kd; ++d) s += (int32_t)q[(size_t)d * N + i] * (int32_t)k[(size_t)d * N + j];
                S[j] = s;
                if (s > mx) mx = s;
            }
            int64_t l = 0;
            for (int d = 0; d < hd; ++d) o[d] = 0;
            for (int j = 0; j < N; ++j) {
                int64_t t = rne((int64_t)(mx - S[j]) * mt, sht);
                const int32_t p = E[t > 255 ? 255 : t];
                l += p;
                for (int d = 0; d < hd; ++d) o[d] += (int64_t)p * v[(size_t)d * N + j];
            }
            for (int d = 0; d < hd; ++d) {
                const int ch = h * hd + d;
                const int64_t a = div_rne(rne(o[d] * mo, sho), l);
                /* positional term of channel ch at pixel i */
                q8 vch = q8_view(&qkv, h * blk + 2 * kd + d, 1);
                const int64_t pe =
                    rne(acc_at(&pq[ch], &vch, 0, i / in->w, i % in->w, 1, 1) * pq[ch].mult[0], pq[ch].shift[0]);
                ope->d[(size_t)ch * N + i] = (int8_t)clampi(a + pe, -127, 127);
            }
        }
        free(o);
        free(S);
        }
    }
    q8_set_scale(ope, s_ope);
    for (int ch = 0; ch < dim; ++ch)
        if (pq[ch].wq) qconv_free(&pq[ch]);
    free(pq);
    q8_free(&qkv);
    return st;
}

static int qpsablock(const i8ctx* x, const char* P, int heads, q8* out, const q8* in) {
    char nm[220];
    const int cf = wdim0(x, "%s.ffn.0.conv.weight", P);
    if (!cf) return I8_ERR_MISSING;
    q8 ope = q8_new(in->c, in->h, in->w), x1 = q8_new(in->c, in->h, in->w), f = q8_new(cf, in->h, in->w);
    int st = qattention(x, P, heads, &ope, in);
    snprintf(nm, sizeof nm, "%s.attn.proj", P);
    if (st == I8_OK) st = qconv(x, nm, &x1, &ope, 1, 0, 0, in);
    snprintf(nm, sizeof nm, "%s.ffn.0", P);
    if (st == I8_OK) st = qconv(x, nm, &f, &x1, 1, 0, 1, NULL);
    snprintf(nm, sizeof nm, "%s.ffn.1", P);
    if (st == I8_OK) st = qconv(x, nm, out, &f, 1, 0, 0, &x1);
    q8_free(&ope);
    q8_free(&x1);
    q8_free(&f);
    return st;
}

static int qc2psa(const i8ctx* x, const char* L, q8* out, const q8* in) {
    char nm[220];
    const int ch = (int)((float)in->c * 0.5f);
    int heads = ch / 64;
    if (heads < 1) heads = 1;
    q8 cat = q8_new(2 * ch, in->h, in->w);
    snprintf(nm, sizeof nm, "%s.cv1", L);
    int st = qconv(x, nm, &cat, in, 1, 0, 1, NULL);
    q8 b = q8_view(&cat, ch, ch);
    q8 t = q8_new(ch, in->h, in->w);
    snprintf(nm, sizeof nm, "%s.m.0", L);
    if (st == I8_OK) st = qpsablock(x, nm, heads, &t, &b);
    if (st == I8_OK) q8_copy(&b, &t);
    snprintf(nm, sizeof nm, "%s.cv2", L);
    if (st == I8_OK) st = qconv(x, nm, out, &cat, 1, 0, 1, NULL);
    q8_free(&t);
    q8_free(&cat);
    return st;
}

static int qc3k2_attn(const i8ctx* x, const char* L, q8* out, const q8* in) {
    char nm[220];
    const int ch = wdim0(x, "%s.cv1.conv.weight", L) / 2;
    if (!ch) return I8_ERR_MISSING;
    q8 cat = q8_new(3 * ch, in->h, in->w);
    q8 a = q8_view(&cat, 0, 2 * ch);
    snprintf(nm, sizeof nm, "%s.cv1", L);
    int st = qconv(x, nm, &a, in, 1, 0, 1, NULL);
    q8 b = q8_view(&cat, ch, ch);
    q8 bo = q8_new(ch, in->h, in->w);
    snprintf(nm, sizeof nm, "%s.m.0.0", L);
    if (st == I8_OK) st = qbottleneck(x, nm, &bo, &b, 1);
    q8 ps = q8_view(&cat, 2 * ch, ch);
    int heads = ch / 64;
    if (heads < 1) heads = 1;
    snprintf(nm, sizeof nm, "%s.m.0.1", L);
    if (st == I8_OK) st = qpsablock(x, nm, heads, &ps, &bo);
    snprintf(nm, sizeof nm, "%s.cv2", L);
    if (st == I8_OK) st = qconv(x, nm, out, &cat, 1, 0, 1, NULL);
    q8_free(&bo);
    q8_free(&cat);
    return st;
}

static q8 qupsample2(const q8* in) {
    q8 o = q8_new(in->c, in->h * 2, in->w * 2);
    for (int c = 0; c < in->c; ++c) {
        for (int y = 0; y < o.h; ++y)
            for (int xx = 0; xx < o.w; ++xx)
                o.d[((size_t)c * o.h + y) * o.w + xx] = in->d[((size_t)c * in->h + y / 2) * in->w + xx / 2];
        o.cs[c] = in->cs[c];
    }
    return o;
}
static q8 qconcat2(const q8* a, const q8* b) {
    q8 o = q8_new(a->c + b->c, a->h, a->w);
    q8 oa = q8_view(&o, 0, a->c), ob = q8_view(&o, a->c, b->c);
    q8_copy(&oa, a);
    q8_copy(&ob, b);
    return o;
}

static void emit8(i8_stage_cb cb, void* user, const char* name, const q8* f) {
    if (cb) cb(user, name, f->d, f->cs, f->c, f->h, f->w);
}

static int qdetect(const i8ctx* x, const q8* feats[3], int max_det, float* dets, float* logits_out, float* dist_out) {
    const int nc = orc_nc(x->m), strides[3] = {8, 16, 32};
    int d4[4];
    const char* b2 = orc_tensor_ptr(x->m, "model.23.one2one_cv2.0.0.conv.weight", d4) ? "one2one_cv2" : "cv2";
    const char* b3 = b2[0] == 'o' ? "one2one_cv3" : "cv3";
    int N = 0;
    for (int s = 0; s < 3; ++s) N += feats[s]->h * feats[s]->w;
    float* pred = (float*)malloc((size_t)N * (4 + nc) * sizeof(float));
    char nm[200];
    int base = 0, st = I8_OK;
    for (int s = 0; s < 3 && st == I8_OK; ++s) {
        const q8* f = feats[s];
        const int hw = f->h * f->w;
        char p0[200], p1[200];
        snprintf(p0, sizeof p0, "model.23.%s.%d.0", b2, s);
        snprintf(p1, sizeof p1, "model.23.%s.%d.1", b2, s);
        const int c2 = wdim0(x, "%s.conv.weight", p0);
        snprintf(nm, sizeof nm, "model.23.%s.%d.0.1", b3, s);
        const int c3 = wdim0(x, "%s.conv.weight", nm);
        if (!c2 || !c3) {
            st = I8_ERR_MISSING;
            break;
        }
        q8 s1 = q8_new(c2, f->h, f->w), s2 = q8_new(c2, f->h, f->w);
        float* box = (float*)malloc((size_t)4 * hw * sizeof(float));
        float* cls = (float*)malloc((size_t)nc * hw * sizeof(float));
        st = qconv(x, p0, &s1, f, 1, 1, 1, NULL);
        if (st == I8_OK) st = qconv(x, p1, &s2, &s1, 1, 1, 1, NULL);
        snprintf(nm, sizeof nm, "model.23.%s.%d.2", b2, s);
        if (st == I8_OK) st = qconv_deq(x, nm, box, &s2);
        q8 d0 = q8_new(f->c, f->h, f->w), pp0 = q8_new(c3, f->h, f->w), d1 = q8_new(c3, f->h, f->w),
           pp1 = q8_new(c3, f->h, f->w);
        snprintf(nm, sizeof nm, "model.23.%s.%d.0.0", b3, s);
        if (st == I8_OK) st = qdw(x, nm, &d0, f);
        snprintf(nm, sizeof nm, "model.23.%s.%d.0.1", b3, s);
        if (st == I8_OK) st = qconv(x, nm, &pp0, &d0, 1, 0, 1, NULL);
        snprintf(nm, sizeof nm, "model.23.%s.%d.1.0", b3, s);
        if (st == I8_OK) st = qdw(x, nm, &d1, &pp0);
        snprintf(nm, sizeof nm, "model.23.%s.%d.1.1", b3, s);
        if (st == I8_OK) st = qconv(x, nm, &pp1, &d1, 1, 0, 1, NULL);
        snprintf(nm, sizeof nm, "model.23.%s.%d.2", b3, s);
        if (st == I8_OK) st = qconv_deq(x, nm, cls, &pp1);
        for (int j = 0; j < hw && st == I8_OK; ++j) {
            const int gy = j / f->w, gx = j % f->w;
            const float ax = (float)gx + 0.5f, ay = (float)gy + 0.5f, sf = (float)strides[s];
            float* r = pred + (size_t)(base + j) * (4 + nc);
            r[0] = (ax - box[0 * hw + j]) * sf;
            r[1] = (ay - box[1 * hw + j]) * sf;
            r[2] = (ax + box[2 * hw + j]) * sf;
            r[3] = (ay + box[3 * hw + j]) * sf;
            if (dist_out)
                for (int u = 0; u < 4; ++u) dist_out[(size_t)(base + j) * 4 + u] = box[u * hw + j];
            for (int c = 0; c < nc; ++c) {
                const float v = cls[(size_t)c * hw + j];
                if (logits_out) logits_out[(size_t)(base + j) * nc + c] = v;
                r[4 + c] = 1.0f / (1.0f + expf(-v));
            }
        }
        q8_free(&s1);
        q8_free(&s2);
        q8_free(&d0);
        q8_free(&pp0);
        q8_free(&d1);
        q8_free(&pp1);
        free(box);
        free(cls);
        base += hw;
    }
    if (st == I8_OK) st = orc_postprocess(pred, N, nc, max_det, max_det, dets);
    free(pred);
    return st;
}

/* Full INT8 forward of one image in [3,H,W] fp32.  names/scales: the scale
 * table.  Outputs dets [max_det][6], logits [N][nc], dist [N][4] (both
 * nullable); cb (nullable) receives the int8 stage tensors 01-23. */
int orc_i8_forward(void* h, const char* const* names, const float* scales, int n_scales, const float* in, int H, int W,
                   int max_det, float* dets, float* logits, float* dist, i8_stage_cb cb, void* user) {
    const i8ctx x = {h, names, scales, n_scales};
    const float s_in = scale_of(&x, "input");
    if (!(s_in > 0.0f)) return I8_ERR_SCALE;
    q8 xi = q8_new(3, H, W);
    for (size_t i = 0; i < (size_t)3 * H * W; ++i) {
        const float v = nearbyintf(in[i] / s_in);
        xi.d[i] = (int8_t)(v < -127.0f ? -127 : v > 127.0f ? 127 : (int)v);
    }
    q8_set_scale(&xi, s_in);
    q8 b[24];
    memset(b, 0, sizeof b);
    int st = I8_OK;
    char p_[32];
#define QDOWN(i, src)                                                               \
    do {                                                                            \
        snprintf(p_, sizeof p_, "model.%d", i);                                     \
        b[i] = q8_new(wdim0(&x, "%s.conv.weight", p_), (src)->h / 2, (src)->w / 2); \
        if (st == I8_OK) st = qconv(&x, p_, &b[i], (src), 2, 1, 1, NULL);           \
    } while (0)
#define QOUT(L) wdim0(&x, "%s.cv2.conv.weight", L)
    QDOWN(0, &xi);
    emit8(cb, user, "stage_01_buf0", &b[0]);
    QDOWN(1, &b[0]);
    emit8(cb, user, "stage_02_buf1", &b[1]);
    b[2] = q8_new(QOUT("model.2"), b[1].h, b[1].w);
    if (st == I8_OK) st = qc3k2_plain(&x, "model.2", 1, 1, &b[2], &b[1]);
    emit8(cb, user, "stage_03_buf2", &b[2]);
    QDOWN(3, &b[2]);
    emit8(cb, user, "stage_04_buf3", &b[3]);
    b[4] = q8_new(QOUT("model.4"), b[3].h, b[3].w);
    if (st == I8_OK) st = qc3k2_plain(&x, "model.4", 1, 1, &b[4], &b[3]);
    emit8(cb, user, "stage_05_buf4", &b[4]);
    QDOWN(5, &b[4]);
    emit8(cb, user, "stage_06_buf5", &b[5]);
    b[6] = q8_new(QOUT("model.6"), b[5].h, b[5].w);
    if (st == I8_OK) st = qc3k2_c3k(&x, "model.6", &b[6], &b[5]);
    emit8(cb, user, "stage_07_buf6", &b[6]);
    QDOWN(7, &b[6]);
    emit8(cb, user, "stage_08_buf7", &b[7]);
    b[8] = q8_new(QOUT("model.8"), b[7].h, b[7].w);
    if (st == I8_OK) st = qc3k2_c3k(&x, "model.8", &b[8], &b[7]);
    emit8(cb, user, "stage_09_buf8", &b[8]);
    b[9] = q8_new(QOUT("model.9"), b[8].h, b[8].w);
    if (st == I8_OK) st = qsppf(&x, "model.9", 5, 3, 1, &b[9], &b[8]);
    emit8(cb, user, "stage_10_buf9", &b[9]);
    b[10] = q8_new(QOUT("model.10"), b[9].h, b[9].w);
    if (st == I8_OK) st = qc2psa(&x, "model.10", &b[10], &b[9]);
    emit8(cb, user, "stage_11_buf10", &b[10]);
    b[11] = qupsample2(&b[10]);
    emit8(cb, user, "stage_12_buf11", &b[11]);
    b[12] = qconcat2(&b[11], &b[6]);
    emit8(cb, user, "stage_13_buf12", &b[12]);
    b[13] = q8_new(QOUT("model.13"), b[12].h, b[12].w);
    if (st == I8_OK) st = qc3k2_c3k(&x, "model.13", &b[13], &b[12]);
    emit8(cb, user, "stage_14_buf13", &b[13]);
    b[14] = qupsample2(&b[13]);
    emit8(cb, user, "stage_15_buf14", &b[14]);
    b[15] = qconcat2(&b[14], &b[4]);
    emit8(cb, user, "stage_16_buf15", &b[15]);
    b[16] = q8_new(QOUT("model.16"), b[15].h, b[15].w);
    if (st == I8_OK) st = qc3k2_c3k(&x, "model.16", &b[16], &b[15]);
    emit8(cb, user, "stage_17_buf16", &b[16]);
    QDOWN(17, &b[16]);
    emit8(cb, user, "stage_18_buf17", &b[17]);
    b[18] = qconcat2(&b[17], &b[13]);
    emit8(cb, user, "stage_19_buf18", &b[18]);
    b[19] = q8_new(QOUT("model.19"), b[18].h, b[18].w);
    if (st == I8_OK) st = qc3k2_c3k(&x, "model.19", &b[19], &b[18]);
    emit8(cb, user, "stage_20_buf19", &b[19]);
    QDOWN(20, &b[19]);
    emit8(cb, user, "stage_21_buf20", &b[20]);
    b[21] = qconcat2(&b[20], &b[10]);
    emit8(cb, user, "stage_22_buf21", &b[21]);
    b[22] = q8_new(QOUT("model.22"), b[21].h, b[21].w);
    if (st == I8_OK) st = qc3k2_attn(&x, "model.22", &b[22], &b[21]);
    emit8(cb, user, "stage_23_buf22", &b[22]);
    if (st == I8_OK) {
        const q8* feats[3] = {&b[16], &b[19], &b[22]};
        st = qdetect(&x, feats, max_det, dets, logits, dist);
    }
    for (int i = 0; i < 23; ++i) q8_free(&b[i]);
    q8_free(&xi);
#undef QDOWN
#undef QOUT
    return st;
}
