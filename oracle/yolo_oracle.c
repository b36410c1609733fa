/*
 * CPU oracle for the YOLO26 path -- TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C restatement of the reference's FP32 forward (phucb2/yolo-baremetal
 * src/layers.c, src/model.c, src/detect.c, src/utils.c), used by tests/,
 * __graft_entry__.smoke() and bench.py's CPU baseline leg as the checker of
 * the CUDA path.  Nothing in the product links or calls it.
 *
 * Pinned by the tests against (a) the reference's own golden fixtures
 * (tests/data/{c3k2_unit,c3k2_yaml,sppf_test,sppf_shortcut,c2psa_test,
 * conv_test}.bin, copied under tests/golden/) and (b) the reference itself,
 * compiled from its sources into oracle/_ref/ by oracle/Makefile and run on
 * the same seeded weights and inputs, stage by stage.
 *
 * Layout: NCHW float32, batch 1 per call (the reference is batch-1 only).
 * Arithmetic order follows the reference loops so the two agree to float
 * rounding: direct convolution sums bias first then ci, ky, kx
 * (layers.c:60-79); 1x1 stride-1 convolutions accumulate over ci with fused
 * multiply-add, then add the bias (the AVX2/FMA tensor_gemm path,
 * tensor.c:64-113 and layers.c:48-58).  Top-k uses the explicit total order
 * (score desc, index asc), which is what the reference's stable glibc qsort
 * produces (detect.c:63-166).
 */
#include <float.h>
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

typedef struct {
    char name[128];
    int dims[4];
    float* data;
} orc_tensor;

typedef struct {
    char name[96];
    float v;
} orc_stat;

typedef struct {
    orc_tensor* t;
    int n, cap;
    int nc;
    /* Calibration statistics (max |x| per named tensor) when stats_on. */
    orc_stat* st;
    int st_n, st_cap, stats_on;
} orc_model;

/* Max |x| of the last conv/dwconv call: before the activation, and of its
 * output (each call reduces its threads' maxima into these after its
 * parallel loop; calls themselves run one at a time). */
static float g_pre_absmax, g_out_absmax;

static void stat_rec(orc_model* m, const char* name, float v) {
    if (!m->stats_on) return;
    for (int i = 0; i < m->st_n; ++i)
        if (strcmp(m->st[i].name, name) == 0) {
            if (v > m->st[i].v) m->st[i].v = v;
            return;
        }
    if (m->st_n == m->st_cap) {
        const int cap = m->st_cap ? 2 * m->st_cap : 256;
        orc_stat* t = (orc_stat*)realloc(m->st, (size_t)cap * sizeof(orc_stat));
        if (!t) return;
        m->st = t;
        m->st_cap = cap;
    }
    snprintf(m->st[m->st_n].name, sizeof m->st[m->st_n].name, "%s", name);
    m->st[m->st_n].v = v;
    m->st_n++;
}

static float absmax_of(const float* d, size_t n) {
    float a = 0.0f;
    for (size_t i = 0; i < n; ++i) {
        const float v = fabsf(d[i]);
        if (v > a) a = v;
    }
    return a;
}

typedef struct {
    float* d;
    int c, h, w;
} fmap;

typedef void (*orc_stage_cb)(void* user, const char* name, const float* data, int n, int c, int h, int w);

enum { ORC_OK = 0, ORC_ERR_MISSING = 5, ORC_ERR_FORMAT = 6, ORC_ERR_DIMS = 2, ORC_ERR_OOM = 3 };

/* ------------------------------------------------------------------ tensors */
static fmap fm_new(int c, int h, int w) {
    fmap f;
    f.c = c;
    f.h = h;
    f.w = w;
    f.d = (float*)calloc((size_t)c * h * w, sizeof(float));
    return f;
}
static void fm_free(fmap* f) {
    free(f->d);
    f->d = NULL;
}
static fmap fm_view(const fmap* f, int c0, int c) {
    fmap v;
    v.c = c;
    v.h = f->h;
    v.w = f->w;
    v.d = f->d + (size_t)c0 * f->h * f->w;
    return v;
}

static orc_tensor* find(orc_model* m, const char* name) {
    for (int i = 0; i < m->n; ++i)
        if (strcmp(m->t[i].name, name) == 0) return &m->t[i];
    return NULL;
}
static orc_tensor* findf(orc_model* m, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
#include <stdarg.h>
static orc_tensor* findf(orc_model* m, const char* fmt, ...) {
    char buf[200];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    return find(m, buf);
}

static int add_tensor(orc_model* m, const char* name, const int dims[4], const float* data) {
    if (m->n == m->cap) {
        int nc = m->cap ? m->cap * 2 : 256;
        orc_tensor* t = (orc_tensor*)realloc(m->t, (size_t)nc * sizeof(orc_tensor));
        if (!t) return ORC_ERR_OOM;
        m->t = t;
        m->cap = nc;
    }
    orc_tensor* t = &m->t[m->n];
    memset(t, 0, sizeof(*t));
    strncpy(t->name, name, sizeof(t->name) - 1);
    size_t n = 1;
    for (int d = 0; d < 4; ++d) {
        t->dims[d] = dims[d];
        n *= (size_t)dims[d];
    }
    t->data = (float*)malloc(n * sizeof(float) + 4);
    if (!t->data) return ORC_ERR_OOM;
    if (data) memcpy(t->data, data, n * sizeof(float));
    else memset(t->data, 0, n * sizeof(float));
    m->n++;
    return ORC_OK;
}

static void remove_tensor(orc_model* m, const char* name) {
    for (int i = 0; i < m->n; ++i) {
        if (strcmp(m->t[i].name, name) == 0) {
            free(m->t[i].data);
            memmove(&m->t[i], &m->t[i + 1], (size_t)(m->n - i - 1) * sizeof(orc_tensor));
            m->n--;
            return;
        }
    }
}

/* BatchNorm fold (utils.c:81-106): scale = gamma / sqrtf(var + 1e-5). */
static void fold_all(orc_model* m) {
    char p[160], b[200];
    for (int i = 0; i < m->n; ++i) {
        const char* nm = m->t[i].name;
        size_t ln = strlen(nm), ls = strlen(".conv.weight");
        if (ln <= ls || strcmp(nm + ln - ls, ".conv.weight") != 0) continue;
        memcpy(p, nm, ln - ls);
        p[ln - ls] = '\0';
        orc_tensor* g = findf(m, "%s.bn.weight", p);
        orc_tensor* be = findf(m, "%s.bn.bias", p);
        orc_tensor* mu = findf(m, "%s.bn.running_mean", p);
        orc_tensor* var = findf(m, "%s.bn.running_var", p);
        if (!g || !be || !mu || !var) continue;
        snprintf(b, sizeof b, "%s.conv.bias", p);
        if (!find(m, b)) {
            int bd[4] = {1, m->t[i].dims[0], 1, 1};
            if (add_tensor(m, b, bd, NULL) != ORC_OK) return;
        }
        orc_tensor* w = &m->t[i];
        orc_tensor* cb = find(m, b);
        g = findf(m, "%s.bn.weight", p);
        be = findf(m, "%s.bn.bias", p);
        mu = findf(m, "%s.bn.running_mean", p);
        var = findf(m, "%s.bn.running_var", p);
        const int oc = w->dims[0];
        const size_t per = (size_t)w->dims[1] * w->dims[2] * w->dims[3];
        for (int o = 0; o < oc; ++o) {
            const float scale = g->data[o] / sqrtf(var->data[o] + 1e-5f);
            for (size_t j = 0; j < per; ++j) w->data[(size_t)o * per + j] *= scale;
            cb->data[o] = (cb->data[o] - mu->data[o]) * scale + be->data[o];
        }
        const char* sfx[5] = {"weight", "bias", "running_mean", "running_var", "num_batches_tracked"};
        for (int s = 0; s < 5; ++s) {
            snprintf(b, sizeof b, "%s.bn.%s", p, sfx[s]);
            remove_tensor(m, b);
        }
        i = -1; /* table changed: rescan */
    }
}

/* ------------------------------------------------------------------ layers */
static float silu1(float x) { return x / (1.0f + expf(-x)); }

static void silu(fmap* f) {
    const size_t n = (size_t)f->c * f->h * f->w;
    for (size_t i = 0; i < n; ++i) f->d[i] = silu1(f->d[i]);
}

/* conv2d_forward (layers.c:41-81) + optional SiLU (layers.c:83-90).
 * Output channels run in parallel (OpenMP); every output element still sums
 * its terms in the reference's order, so the result does not depend on the
 * thread count. */
static void conv(fmap* out, const fmap* in, const orc_tensor* w, const orc_tensor* b, int stride, int pad, int act) {
    const int oc = w->dims[0], ic = w->dims[1], kh = w->dims[2], kw = w->dims[3];
    const int H = in->h, W = in->w, Ho = out->h, Wo = out->w;
    float pre_m = 0.0f, out_m = 0.0f;
    if (kh == 1 && kw == 1 && stride == 1 && pad == 0) {
        const int P = H * W;
        /* tensor_gemm's AVX2 loop fuses multiply-add on 16- and 8-wide blocks
         * of columns and leaves a scalar tail computed as multiply then add
         * (tensor.c:83-109, built without FP contraction). */
        const int P16 = (P / 16) * 16;
        const int Pv = P16 + ((P - P16) >= 8 ? 8 : 0);
#pragma omp parallel for schedule(dynamic) reduction(max : pre_m, out_m)
        for (int o = 0; o < oc; ++o) {
            float* y = out->d + (size_t)o * P;
            for (int p = 0; p < P; ++p) y[p] = 0.0f;
            for (int c = 0; c < ic; ++c) {
                const float a = w->data[(size_t)o * ic + c];
                if (a == 0.0f) continue;
                const float* x = in->d + (size_t)c * P;
                for (int p = 0; p < Pv; ++p) y[p] = fmaf(a, x[p], y[p]);
                for (int p = Pv; p < P; ++p) {
                    const float prod = a * x[p];
                    y[p] = y[p] + prod;
                }
            }
            if (b)
                for (int p = 0; p < P; ++p) y[p] += b->data[o];
            for (int p = 0; p < P; ++p)
                if (fabsf(y[p]) > pre_m) pre_m = fabsf(y[p]);
            if (act)
                for (int p = 0; p < P; ++p) y[p] = silu1(y[p]);
            for (int p = 0; p < P; ++p)
                if (fabsf(y[p]) > out_m) out_m = fabsf(y[p]);
        }
    } else {
        /* Direct convolution: the reference sums, per output, the bias and
         * then the products in (ci, ky, kx) order, skipping taps outside the
         * image.  Walking (ci, ky, kx) outermost and the output plane inside
         * adds the same terms to every output in the same order. */
#pragma omp parallel for schedule(dynamic) reduction(max : pre_m, out_m)
        for (int o = 0; o < oc; ++o) {
            float* y = out->d + (size_t)o * Ho * Wo;
            const float bv = b ? b->data[o] : 0.0f;
            for (size_t p = 0; p < (size_t)Ho * Wo; ++p) y[p] = bv;
            for (int c = 0; c < ic; ++c) {
                const float* xc = in->d + (size_t)c * H * W;
                for (int ky = 0; ky < kh; ++ky)
                    for (int kx = 0; kx < kw; ++kx) {
                        const float wv = w->data[(((size_t)o * ic + c) * kh + ky) * kw + kx];
                        const int lo = pad - kx, hi = W - 1 + pad - kx;
                        const int ox0 = lo > 0 ? (lo + stride - 1) / stride : 0;
                        int ox1 = hi >= 0 ? hi / stride + 1 : 0;
                        if (ox1 > Wo) ox1 = Wo;
                        for (int oy = 0; oy < Ho; ++oy) {
                            const int iy = oy * stride - pad + ky;
                            if (iy < 0 || iy >= H) continue;
                            const float* xr = xc + (size_t)iy * W - pad + kx;
                            float* yr = y + (size_t)oy * Wo;
                            for (int ox = ox0; ox < ox1; ++ox) {
                                const float prod = xr[ox * stride] * wv;
                                yr[ox] = yr[ox] + prod;
                            }
                        }
                    }
            }
            for (size_t p = 0; p < (size_t)Ho * Wo; ++p) {
                const float s = y[p];
                const float r = act ? silu1(s) : s;
                if (fabsf(s) > pre_m) pre_m = fabsf(s);
                if (fabsf(r) > out_m) out_m = fabsf(r);
                y[p] = r;
            }
        }
    }
    if (pre_m > g_pre_absmax) g_pre_absmax = pre_m;
    if (out_m > g_out_absmax) g_out_absmax = out_m;
}

/* dwconv3x3_same_forward (layers.c:269-290). */
static void dwconv(fmap* out, const fmap* in, const orc_tensor* w, const orc_tensor* b, int act) {
    const int C = in->c, H = in->h, W = in->w;
    float pre_m = 0.0f, out_m = 0.0f;
#pragma omp parallel for schedule(dynamic) reduction(max : pre_m, out_m)
    for (int c = 0; c < C; ++c) {
        for (int y = 0; y < H; ++y) {
            for (int x = 0; x < W; ++x) {
                float s = b ? b->data[c] : 0.0f;
                for (int ky = 0; ky < 3; ++ky) {
                    const int iy = y - 1 + ky;
                    if (iy < 0 || iy >= H) continue;
                    for (int kx = 0; kx < 3; ++kx) {
                        const int ix = x - 1 + kx;
                        if (ix < 0 || ix >= W) continue;
                        const float prod = in->d[((size_t)c * H + iy) * W + ix] * w->data[(size_t)c * 9 + ky * 3 + kx];
                        s = s + prod;
                    }
                }
                const float r = act ? silu1(s) : s;
                if (fabsf(s) > pre_m) pre_m = fabsf(s);
                if (fabsf(r) > out_m) out_m = fabsf(r);
                out->d[((size_t)c * H + y) * W + x] = r;
            }
        }
    }
    if (pre_m > g_pre_absmax) g_pre_absmax = pre_m;
    if (out_m > g_out_absmax) g_out_absmax = out_m;
}

/* pool2d_max_forward, stride 1, padding k/2 excluded (layers.c:191-217). */
static void maxpool(fmap* out, const fmap* in, int k) {
    const int C = in->c, H = in->h, W = in->w, pad = k / 2;
#pragma omp parallel for schedule(static)
    for (int c = 0; c < C; ++c)
        for (int y = 0; y < H; ++y)
            for (int x = 0; x < W; ++x) {
                float m = -FLT_MAX;
                for (int ky = 0; ky < k; ++ky) {
                    const int iy = y - pad + ky;
                    if (iy < 0 || iy >= H) continue;
                    for (int kx = 0; kx < k; ++kx) {
                        const int ix = x - pad + kx;
                        if (ix < 0 || ix >= W) continue;
                        const float v = in->d[((size_t)c * H + iy) * W + ix];
                        if (v > m) m = v;
                    }
                }
                out->d[((size_t)c * H + y) * W + x] = m;
            }
}

static void add_into(fmap* y, const fmap* x) {
    const size_t n = (size_t)y->c * y->h * y->w;
    for (size_t i = 0; i < n; ++i) y->d[i] += x->d[i];
}

static int conv_named(orc_model* m, const char* prefix, fmap* out, const fmap* in, int stride, int pad, int act) {
    orc_tensor* w = findf(m, "%s.conv.weight", prefix);
    orc_tensor* b = findf(m, "%s.conv.bias", prefix);
    if (!w || !b) return ORC_ERR_MISSING;
    if (w->dims[1] != in->c || w->dims[0] != out->c) return ORC_ERR_DIMS;
    g_pre_absmax = g_out_absmax = 0.0f;
    conv(out, in, w, b, stride, pad, act);
    if (m->stats_on) {
        char nm[120];
        if (act) {
            snprintf(nm, sizeof nm, "%s:pre", prefix);
            stat_rec(m, nm, g_pre_absmax);
        }
        stat_rec(m, prefix, g_out_absmax);
    }
    return ORC_OK;
}

static void stat_map(orc_model* m, const char* name, const fmap* f) {
    if (m->stats_on) stat_rec(m, name, absmax_of(f->d, (size_t)f->c * f->h * f->w));
}

/* Bottleneck (layers.c:92-108). */
static int bottleneck(orc_model* m, const char* p, fmap* out, const fmap* in, int shortcut) {
    char n1[200], n2[200];
    snprintf(n1, sizeof n1, "%s.cv1", p);
    snprintf(n2, sizeof n2, "%s.cv2", p);
    orc_tensor* w1 = findf(m, "%s.conv.weight", n1);
    orc_tensor* w2 = findf(m, "%s.conv.weight", n2);
    if (!w1 || !w2) return ORC_ERR_MISSING;
    fmap t = fm_new(w1->dims[0], in->h, in->w);
    int st = conv_named(m, n1, &t, in, 1, (w1->dims[2] - 1) / 2, 1);
    if (st == ORC_OK) st = conv_named(m, n2, out, &t, 1, (w2->dims[2] - 1) / 2, 1);
    fm_free(&t);
    if (st == ORC_OK && shortcut) {
        add_into(out, in);
        stat_map(m, n2, out);
    }
    return st;
}

/* C3k2 without C3k (layers.c:110-154): cat(a, b, m0(b), ...) -> cv2. */
static int c3k2_plain(orc_model* m, const char* L, int n, int shortcut, fmap* out, const fmap* in) {
    char nm[220];
    orc_tensor* w1 = findf(m, "%s.cv1.conv.weight", L);
    if (!w1) return ORC_ERR_MISSING;
    const int ct = w1->dims[0], ch = ct / 2;
    fmap cat = fm_new((2 + n) * ch, in->h, in->w);
    fmap a = fm_view(&cat, 0, ct);
    snprintf(nm, sizeof nm, "%s.cv1", L);
    int st = conv_named(m, nm, &a, in, 1, 0, 1);
    for (int i = 0; i < n && st == ORC_OK; ++i) {
        fmap prev = fm_view(&cat, i == 0 ? ch : (1 + i) * ch, ch);
        fmap y = fm_view(&cat, (2 + i) * ch, ch);
        snprintf(nm, sizeof nm, "%s.m.%d", L, i);
        st = bottleneck(m, nm, &y, &prev, shortcut);
    }
    snprintf(nm, sizeof nm, "%s.cv2", L);
    if (st == ORC_OK) st = conv_named(m, nm, out, &cat, 1, 0, 1);
    fm_free(&cat);
    return st;
}

/* C3 / C3k (layers.c:156-189): cv3(cat(m(cv1(x)), cv2(x))). */
static int c3(orc_model* m, const char* P, int shortcut, fmap* out, const fmap* in) {
    char nm[220];
    orc_tensor* w1 = findf(m, "%s.cv1.conv.weight", P);
    orc_tensor* w2 = findf(m, "%s.cv2.conv.weight", P);
    if (!w1 || !w2) return ORC_ERR_MISSING;
    const int cm = w1->dims[0], c2 = w2->dims[0];
    fmap cat = fm_new(cm + c2, in->h, in->w);
    fmap y = fm_new(cm, in->h, in->w);
    fmap z = fm_new(cm, in->h, in->w);
    fmap v2 = fm_view(&cat, cm, c2);
    snprintf(nm, sizeof nm, "%s.cv1", P);
    int st = conv_named(m, nm, &y, in, 1, 0, 1);
    snprintf(nm, sizeof nm, "%s.cv2", P);
    if (st == ORC_OK) st = conv_named(m, nm, &v2, in, 1, 0, 1);
    fmap* cur = &y;
    fmap* nxt = &z;
    for (int i = 0; st == ORC_OK; ++i) {
        snprintf(nm, sizeof nm, "%s.m.%d", P, i);
        char probe[240];
        snprintf(probe, sizeof probe, "%s.cv1.conv.weight", nm);
        if (!find(m, probe)) break;
        st = bottleneck(m, nm, nxt, cur, shortcut);
        fmap* t = cur;
        cur = nxt;
        nxt = t;
    }
    memcpy(cat.d, cur->d, (size_t)cm * in->h * in->w * sizeof(float));
    snprintf(nm, sizeof nm, "%s.cv3", P);
    if (st == ORC_OK) st = conv_named(m, nm, out, &cat, 1, 0, 1);
    fm_free(&y);
    fm_free(&z);
    fm_free(&cat);
    return st;
}

/* C3k2 with inner C3k (model.c:415-557). */
/* The reference wires exactly one C3k (m.0); C3k blocks m.1, m.2, ... when
 * present chain on the previous block's output as in the C2f layout
 * (cat(a, b, m0(b), m1(m0(b)), ...) -> cv2), which is identical for n = 1. */
static int c3k2_c3k(orc_model* m, const char* L, fmap* out, const fmap* in) {
    char nm[220];
    orc_tensor* w1 = findf(m, "%s.cv1.conv.weight", L);
    orc_tensor* k3 = findf(m, "%s.m.0.cv3.conv.weight", L);
    if (!w1 || !k3) return ORC_ERR_MISSING;
    const int ch = w1->dims[0] / 2;
    int n = 0;
    while (findf(m, "%s.m.%d.cv3.conv.weight", L, n)) ++n;
    fmap cat = fm_new(2 * ch + n * k3->dims[0], in->h, in->w);
    fmap a = fm_view(&cat, 0, 2 * ch);
    snprintf(nm, sizeof nm, "%s.cv1", L);
    int st = conv_named(m, nm, &a, in, 1, 0, 1);
    for (int i = 0; i < n && st == ORC_OK; ++i) {
        fmap b = fm_view(&cat, i == 0 ? ch : 2 * ch + (i - 1) * k3->dims[0], i == 0 ? ch : k3->dims[0]);
        fmap o = fm_view(&cat, 2 * ch + i * k3->dims[0], k3->dims[0]);
        snprintf(nm, sizeof nm, "%s.m.%d", L, i);
        st = c3(m, nm, 1, &o, &b);
    }
    snprintf(nm, sizeof nm, "%s.cv2", L);
    if (st == ORC_OK) st = conv_named(m, nm, out, &cat, 1, 0, 1);
    fm_free(&cat);
    return st;
}

/* SPPF (layers.c:230-265). */
static int sppf(orc_model* m, const char* L, int k, int n_pool, int shortcut, fmap* out, const fmap* in) {
    char nm[220];
    orc_tensor* w1 = findf(m, "%s.cv1.conv.weight", L);
    if (!w1) return ORC_ERR_MISSING;
    const int c = w1->dims[0];
    fmap cat = fm_new(c * (n_pool + 1), in->h, in->w);
    fmap s0 = fm_view(&cat, 0, c);
    snprintf(nm, sizeof nm, "%s.cv1", L);
    int st = conv_named(m, nm, &s0, in, 1, 0, 0);
    for (int j = 0; j < n_pool && st == ORC_OK; ++j) {
        fmap a = fm_view(&cat, j * c, c), b = fm_view(&cat, (j + 1) * c, c);
        maxpool(&b, &a, k);
    }
    snprintf(nm, sizeof nm, "%s.cv2", L);
    if (st == ORC_OK) st = conv_named(m, nm, out, &cat, 1, 0, 1);
    if (st == ORC_OK && shortcut && in->c == out->c) {
        add_into(out, in);
        snprintf(nm, sizeof nm, "%s.cv2", L);
        stat_map(m, nm, out);
    }
    fm_free(&cat);
    return st;
}

/* Attention (layers.c:310-405) with full N x N logits, as the reference. */
static int attention(orc_model* m, const char* P, int heads, float ratio, fmap* out, const fmap* in) {
    char nm[220];
    const int dim = in->c, N = in->h * in->w;
    if (dim % heads) return ORC_ERR_DIMS;
    const int hd = dim / heads, kd = (int)((float)hd * ratio);
    const float scale = powf((float)kd, -0.5f);
    orc_tensor* wq = findf(m, "%s.attn.qkv.conv.weight", P);
    orc_tensor* pe_w = findf(m, "%s.attn.pe.conv.weight", P);
    orc_tensor* pe_b = findf(m, "%s.attn.pe.conv.bias", P);
    if (!wq || !pe_w || !pe_b) return ORC_ERR_MISSING;
    if (wq->dims[0] != dim + 2 * kd * heads) return ORC_ERR_DIMS;
    fmap qkv = fm_new(wq->dims[0], in->h, in->w);
    snprintf(nm, sizeof nm, "%s.attn.qkv", P);
    int st = conv_named(m, nm, &qkv, in, 1, 0, 0);
    fmap ao = fm_new(dim, in->h, in->w);
    fmap vpe = fm_new(dim, in->h, in->w);
    const int blk = 2 * kd + hd;
    for (int h = 0; h < heads && st == ORC_OK; ++h) {
        const float* q = qkv.d + (size_t)(h * blk) * N;
        const float* k = qkv.d + (size_t)(h * blk + kd) * N;
        const float* v = qkv.d + (size_t)(h * blk + 2 * kd) * N;
        float* S = (float*)malloc((size_t)N * N * sizeof(float));
#pragma omp parallel for schedule(static)
        for (int i = 0; i < N; ++i) {
            float* row = S + (size_t)i * N;
            for (int j = 0; j < N; ++j) {
                float s = 0.0f;
                for (int d = 0; d < kd; ++d) s += q[(size_t)d * N + i] * k[(size_t)d * N + j];
                row[j] = s * scale;
            }
            float mx = row[0];
            for (int j = 1; j < N; ++j)
                if (row[j] > mx) mx = row[j];
            float sum = 0.0f;
            for (int j = 0; j < N; ++j) {
                row[j] = expf(row[j] - mx);
                sum += row[j];
            }
            if (sum > 1e-12f)
                for (int j = 0; j < N; ++j) row[j] /= sum;
        }
#pragma omp parallel for schedule(static)
        for (int d = 0; d < hd; ++d)
            for (int j = 0; j < N; ++j) {
                float s = 0.0f;
                for (int t = 0; t < N; ++t) s += v[(size_t)d * N + t] * S[(size_t)j * N + t];
                ao.d[(size_t)(h * hd + d) * N + j] = s;
            }
        memcpy(vpe.d + (size_t)h * hd * N, v, (size_t)hd * N * sizeof(float));
        free(S);
    }
    fmap pe = fm_new(dim, in->h, in->w);
    dwconv(&pe, &vpe, pe_w, pe_b, 0);
    add_into(&ao, &pe);
    snprintf(nm, sizeof nm, "%s.attn.ope", P);
    stat_map(m, nm, &ao);
    snprintf(nm, sizeof nm, "%s.attn.proj", P);
    if (st == ORC_OK) st = conv_named(m, nm, out, &ao, 1, 0, 0);
    fm_free(&pe);
    fm_free(&vpe);
    fm_free(&ao);
    fm_free(&qkv);
    return st;
}

/* PSABlock (layers.c:407-453): x1 = x + attn(x); out = x1 + ffn(x1). */
static int psablock(orc_model* m, const char* P, int heads, float ratio, int shortcut, fmap* out, const fmap* in) {
    char nm[220];
    orc_tensor* f0 = findf(m, "%s.ffn.0.conv.weight", P);
    if (!f0) return ORC_ERR_MISSING;
    fmap x1 = fm_new(in->c, in->h, in->w);
    int st = attention(m, P, heads, ratio, &x1, in);
    if (st == ORC_OK && shortcut) {
        add_into(&x1, in);
        snprintf(nm, sizeof nm, "%s.attn.proj", P);
        stat_map(m, nm, &x1);
    }
    fmap f = fm_new(f0->dims[0], in->h, in->w);
    snprintf(nm, sizeof nm, "%s.ffn.0", P);
    if (st == ORC_OK) st = conv_named(m, nm, &f, &x1, 1, 0, 1);
    snprintf(nm, sizeof nm, "%s.ffn.1", P);
    if (st == ORC_OK) st = conv_named(m, nm, out, &f, 1, 0, 0);
    if (st == ORC_OK && shortcut) {
        add_into(out, &x1);
        snprintf(nm, sizeof nm, "%s.ffn.1", P);
        stat_map(m, nm, out);
    }
    fm_free(&f);
    fm_free(&x1);
    return st;
}

/* C2PSA (layers.c:455-496). */
static int c2psa(orc_model* m, const char* L, int n_blocks, float e, float ratio, fmap* out, const fmap* in) {
    char nm[220];
    const int ch = (int)((float)in->c * e);
    int heads = ch / 64;
    if (heads < 1) heads = 1;
    fmap cat = fm_new(2 * ch, in->h, in->w);
    snprintf(nm, sizeof nm, "%s.cv1", L);
    int st = conv_named(m, nm, &cat, in, 1, 0, 1);
    fmap b = fm_view(&cat, ch, ch);
    fmap t = fm_new(ch, in->h, in->w);
    for (int i = 0; i < n_blocks && st == ORC_OK; ++i) {
        snprintf(nm, sizeof nm, "%s.m.%d", L, i);
        st = psablock(m, nm, heads, ratio, 1, &t, &b);
        memcpy(b.d, t.d, (size_t)ch * in->h * in->w * sizeof(float));
    }
    snprintf(nm, sizeof nm, "%s.cv2", L);
    if (st == ORC_OK) st = conv_named(m, nm, out, &cat, 1, 0, 1);
    fm_free(&t);
    fm_free(&cat);
    return st;
}

/* Head C3k2 with Bottleneck + PSABlock (model.c:560-665). */
static int c3k2_attn(orc_model* m, const char* L, fmap* out, const fmap* in) {
    char nm[220];
    orc_tensor* w1 = findf(m, "%s.cv1.conv.weight", L);
    if (!w1) return ORC_ERR_MISSING;
    const int ch = w1->dims[0] / 2;
    fmap cat = fm_new(3 * ch, in->h, in->w);
    fmap a = fm_view(&cat, 0, 2 * ch);
    snprintf(nm, sizeof nm, "%s.cv1", L);
    int st = conv_named(m, nm, &a, in, 1, 0, 1);
    fmap b = fm_view(&cat, ch, ch);
    fmap bo = fm_new(ch, in->h, in->w);
    snprintf(nm, sizeof nm, "%s.m.0.0", L);
    if (st == ORC_OK) st = bottleneck(m, nm, &bo, &b, 1);
    fmap ps = fm_view(&cat, 2 * ch, ch);
    int heads = ch / 64;
    if (heads < 1) heads = 1;
    snprintf(nm, sizeof nm, "%s.m.0.1", L);
    if (st == ORC_OK) st = psablock(m, nm, heads, 0.5f, 1, &ps, &bo);
    snprintf(nm, sizeof nm, "%s.cv2", L);
    if (st == ORC_OK) st = conv_named(m, nm, out, &cat, 1, 0, 1);
    fm_free(&bo);
    fm_free(&cat);
    return st;
}

static fmap upsample2(const fmap* in) {
    fmap o = fm_new(in->c, in->h * 2, in->w * 2);
    for (int c = 0; c < in->c; ++c)
        for (int y = 0; y < o.h; ++y)
            for (int x = 0; x < o.w; ++x)
                o.d[((size_t)c * o.h + y) * o.w + x] = in->d[((size_t)c * in->h + y / 2) * in->w + x / 2];
    return o;
}
static fmap concat2(const fmap* a, const fmap* b) {
    fmap o = fm_new(a->c + b->c, a->h, a->w);
    memcpy(o.d, a->d, (size_t)a->c * a->h * a->w * sizeof(float));
    memcpy(o.d + (size_t)a->c * a->h * a->w, b->d, (size_t)b->c * b->h * b->w * sizeof(float));
    return o;
}

/* ----------------------------------------------------------------- top-k */
typedef struct {
    float v;
    int i;
} kv_t;
static int kv_cmp(const void* pa, const void* pb) {
    const kv_t* a = (const kv_t*)pa;
    const kv_t* b = (const kv_t*)pb;
    if (a->v > b->v) return -1;
    if (a->v < b->v) return 1;
    return (a->i > b->i) - (a->i < b->i);
}

/* detect_postprocess_from_pred (detect.c:63-166) with explicit tie order. */
int orc_postprocess(const float* pred, int N, int nc, int max_det, int cap, float* out) {
    int k = max_det < N ? max_det : N;
    if (k > cap) k = cap;
    kv_t* a = (kv_t*)malloc((size_t)(N > 0 ? N : 1) * sizeof(kv_t));
    for (int j = 0; j < N; ++j) {
        float mx = -FLT_MAX;
        for (int c = 0; c < nc; ++c) {
            const float v = pred[(size_t)j * (4 + nc) + 4 + c];
            if (v > mx) mx = v;
        }
        a[j].v = mx;
        a[j].i = j;
    }
    qsort(a, (size_t)N, sizeof(kv_t), kv_cmp);
    kv_t* f = (kv_t*)malloc((size_t)(k > 0 ? k : 1) * nc * sizeof(kv_t));
    for (int s = 0; s < k; ++s)
        for (int c = 0; c < nc; ++c) {
            f[(size_t)s * nc + c].v = pred[(size_t)a[s].i * (4 + nc) + 4 + c];
            f[(size_t)s * nc + c].i = s * nc + c;
        }
    qsort(f, (size_t)k * nc, sizeof(kv_t), kv_cmp);
    for (int t = 0; t < cap; ++t) {
        float* r = out + (size_t)t * 6;
        if (t < k) {
            const int slot = f[t].i / nc, c = f[t].i % nc;
            const float* br = pred + (size_t)a[slot].i * (4 + nc);
            r[0] = br[0];
            r[1] = br[1];
            r[2] = br[2];
            r[3] = br[3];
            r[4] = f[t].v;
            r[5] = (float)c;
        } else {
            for (int u = 0; u < 6; ++u) r[u] = 0.0f;
        }
    }
    free(f);
    free(a);
    return ORC_OK;
}

/* Detect one2one (detect.c:253-454).  logits_out [N, nc] anchor-major and
 * boxes_out [N, 4] are optional. */
static int detect(orc_model* m, const fmap* feats[3], int max_det, float* dets, float* logits_out, float* boxes_out) {
    const int nc = m->nc, strides[3] = {8, 16, 32};
    const char* b2 = findf(m, "model.23.one2one_cv2.0.0.conv.weight") ? "one2one_cv2" : "cv2";
    const char* b3 = b2[0] == 'o' ? "one2one_cv3" : "cv3";
    int N = 0;
    for (int s = 0; s < 3; ++s) N += feats[s]->h * feats[s]->w;
    float* pred = (float*)malloc((size_t)N * (4 + nc) * sizeof(float));
    char nm[200];
    int base = 0, st = ORC_OK;
    for (int s = 0; s < 3 && st == ORC_OK; ++s) {
        const fmap* f = feats[s];
        const int hw = f->h * f->w;
        orc_tensor* w0 = findf(m, "model.23.%s.%d.0.conv.weight", b2, s);
        orc_tensor* pw = findf(m, "model.23.%s.%d.0.1.conv.weight", b3, s);
        orc_tensor* w2 = findf(m, "model.23.%s.%d.2.weight", b2, s);
        orc_tensor* bb2 = findf(m, "model.23.%s.%d.2.bias", b2, s);
        orc_tensor* wf = findf(m, "model.23.%s.%d.2.weight", b3, s);
        orc_tensor* bf = findf(m, "model.23.%s.%d.2.bias", b3, s);
        orc_tensor* dw0 = findf(m, "model.23.%s.%d.0.0.conv.weight", b3, s);
        orc_tensor* db0 = findf(m, "model.23.%s.%d.0.0.conv.bias", b3, s);
        orc_tensor* dw1 = findf(m, "model.23.%s.%d.1.0.conv.weight", b3, s);
        orc_tensor* db1 = findf(m, "model.23.%s.%d.1.0.conv.bias", b3, s);
        if (!w0 || !pw || !w2 || !bb2 || !wf || !bf || !dw0 || !db0 || !dw1 || !db1) {
            st = ORC_ERR_MISSING;
            break;
        }
        const int c2 = w0->dims[0], c3 = pw->dims[0];
        fmap s1 = fm_new(c2, f->h, f->w), s2 = fm_new(c2, f->h, f->w), box = fm_new(4, f->h, f->w);
        snprintf(nm, sizeof nm, "model.23.%s.%d.0", b2, s);
        st = conv_named(m, nm, &s1, f, 1, 1, 1);
        snprintf(nm, sizeof nm, "model.23.%s.%d.1", b2, s);
        if (st == ORC_OK) st = conv_named(m, nm, &s2, &s1, 1, 1, 1);
        if (st == ORC_OK) conv(&box, &s2, w2, bb2, 1, 0, 0);
        fmap d0 = fm_new(f->c, f->h, f->w), p0 = fm_new(c3, f->h, f->w), d1 = fm_new(c3, f->h, f->w),
             p1 = fm_new(c3, f->h, f->w), cls = fm_new(nc, f->h, f->w);
        g_pre_absmax = g_out_absmax = 0.0f;
        if (st == ORC_OK) dwconv(&d0, f, dw0, db0, 1);
        snprintf(nm, sizeof nm, "model.23.%s.%d.0.0:pre", b3, s);
        stat_rec(m, nm, g_pre_absmax);
        snprintf(nm, sizeof nm, "model.23.%s.%d.0.0", b3, s);
        stat_rec(m, nm, g_out_absmax);
        snprintf(nm, sizeof nm, "model.23.%s.%d.0.1", b3, s);
        if (st == ORC_OK) st = conv_named(m, nm, &p0, &d0, 1, 0, 1);
        g_pre_absmax = g_out_absmax = 0.0f;
        if (st == ORC_OK) dwconv(&d1, &p0, dw1, db1, 1);
        snprintf(nm, sizeof nm, "model.23.%s.%d.1.0:pre", b3, s);
        stat_rec(m, nm, g_pre_absmax);
        snprintf(nm, sizeof nm, "model.23.%s.%d.1.0", b3, s);
        stat_rec(m, nm, g_out_absmax);
        snprintf(nm, sizeof nm, "model.23.%s.%d.1.1", b3, s);
        if (st == ORC_OK) st = conv_named(m, nm, &p1, &d1, 1, 0, 1);
        if (st == ORC_OK) conv(&cls, &p1, wf, bf, 1, 0, 0);
        for (int j = 0; j < hw && st == ORC_OK; ++j) {
            const int gy = j / f->w, gx = j % f->w;
            const float ax = (float)gx + 0.5f, ay = (float)gy + 0.5f, sf = (float)strides[s];
            float* r = pred + (size_t)(base + j) * (4 + nc);
            r[0] = (ax - box.d[0 * hw + j]) * sf;
            r[1] = (ay - box.d[1 * hw + j]) * sf;
            r[2] = (ax + box.d[2 * hw + j]) * sf;
            r[3] = (ay + box.d[3 * hw + j]) * sf;
            for (int c = 0; c < nc; ++c) {
                const float x = cls.d[(size_t)c * hw + j];
                if (logits_out) logits_out[(size_t)(base + j) * nc + c] = x;
                r[4 + c] = 1.0f / (1.0f + expf(-x));
            }
            if (boxes_out)
                for (int u = 0; u < 4; ++u) boxes_out[(size_t)(base + j) * 4 + u] = r[u];
        }
        fm_free(&s1);
        fm_free(&s2);
        fm_free(&box);
        fm_free(&d0);
        fm_free(&p0);
        fm_free(&d1);
        fm_free(&p1);
        fm_free(&cls);
        base += hw;
    }
    if (st == ORC_OK) st = orc_postprocess(pred, N, nc, max_det, max_det, dets);
    free(pred);
    return st;
}

/* ------------------------------------------------------------------ public */
void* orc_new(int nc) {
    orc_model* m = (orc_model*)calloc(1, sizeof(orc_model));
    if (m) m->nc = nc;
    return m;
}

void orc_free(void* h) {
    orc_model* m = (orc_model*)h;
    if (!m) return;
    for (int i = 0; i < m->n; ++i) free(m->t[i].data);
    free(m->t);
    free(m->st);
    free(m);
}

int orc_add(void* h, const char* name, const int* dims4, const float* data) {
    return add_tensor((orc_model*)h, name, dims4, data);
}

void orc_fold(void* h) { fold_all((orc_model*)h); }

int orc_num_tensors(void* h) { return ((orc_model*)h)->n; }

/* Copies a (folded) tensor out; returns its element count, or -1. */
long orc_get(void* h, const char* name, float* out, long cap) {
    orc_tensor* t = find((orc_model*)h, name);
    if (!t) return -1;
    const long n = (long)t->dims[0] * t->dims[1] * t->dims[2] * t->dims[3];
    if (out && cap >= n) memcpy(out, t->data, (size_t)n * sizeof(float));
    return n;
}

/* Reads a converter-layout .bin and folds BatchNorm. */
void* orc_load(const char* path) {
    FILE* f = fopen(path, "rb");
    if (!f) return NULL;
    int32_t nc = 0, count = 0;
    if (fread(&nc, 4, 1, f) != 1 || fread(&count, 4, 1, f) != 1) {
        fclose(f);
        return NULL;
    }
    orc_model* m = (orc_model*)orc_new(nc);
    for (int i = 0; i < count; ++i) {
        int32_t nl = 0, nd = 0, dims[4] = {1, 1, 1, 1};
        char name[128];
        if (fread(&nl, 4, 1, f) != 1 || nl <= 0 || nl >= 128 || fread(name, 1, (size_t)nl, f) != (size_t)nl ||
            fread(&nd, 4, 1, f) != 1 || nd < 0 || nd > 4) {
            fclose(f);
            orc_free(m);
            return NULL;
        }
        name[nl] = '\0';
        for (int d = 0; d < nd; ++d)
            if (fread(&dims[d], 4, 1, f) != 1) {
                fclose(f);
                orc_free(m);
                return NULL;
            }
        if (add_tensor(m, name, dims, NULL) != ORC_OK) {
            fclose(f);
            orc_free(m);
            return NULL;
        }
        const size_t n = (size_t)dims[0] * dims[1] * dims[2] * dims[3];
        if (fread(m->t[m->n - 1].data, 4, n, f) != n) {
            fclose(f);
            orc_free(m);
            return NULL;
        }
    }
    fclose(f);
    fold_all(m);
    return m;
}

/* Calibration statistics: on != 0 clears the table and starts recording
 * max |x| per named tensor over the following forwards. */
void orc_stats_enable(void* h, int on) {
    orc_model* m = (orc_model*)h;
    m->stats_on = on;
    if (on) m->st_n = 0;
}
int orc_stats_count(void* h) { return ((orc_model*)h)->st_n; }
int orc_stats_entry(void* h, int i, char* name, int cap, float* v) {
    orc_model* m = (orc_model*)h;
    if (i < 0 || i >= m->st_n) return -1;
    snprintf(name, (size_t)cap, "%s", m->st[i].name);
    *v = m->st[i].v;
    return 0;
}

/* Pointer to a (folded) tensor's data and its dims, or NULL. */
const float* orc_tensor_ptr(void* h, const char* name, int* dims4) {
    orc_tensor* t = find((orc_model*)h, name);
    if (!t) return NULL;
    if (dims4)
        for (int d = 0; d < 4; ++d) dims4[d] = t->dims[d];
    return t->data;
}
int orc_nc(void* h) { return ((orc_model*)h)->nc; }

int orc_anchors(int H, int W) { return (H / 8) * (W / 8) + (H / 16) * (W / 16) + (H / 32) * (W / 32); }

static void emit(orc_stage_cb cb, void* user, const char* name, const fmap* f) {
    if (cb) cb(user, name, f->d, 1, f->c, f->h, f->w);
}

/* Full forward of one image (model.c:764-903). */
int orc_forward(void* h, const float* in, int H, int W, int max_det, float* dets, float* logits, float* boxes,
                orc_stage_cb cb, void* user) {
    orc_model* m = (orc_model*)h;
    fmap x;
    x.c = 3;
    x.h = H;
    x.w = W;
    x.d = (float*)in;
    emit(cb, user, "stage_00_input", &x);
    stat_map(m, "input", &x);
    fmap b[24];
    memset(b, 0, sizeof b);
    int st = ORC_OK;
#define WID(name) (findf(m, "%s.conv.weight", name) ? findf(m, "%s.conv.weight", name)->dims[0] : 0)
#define DOWN(i, src)                                                      \
    do {                                                                  \
        char p_[32];                                                      \
        snprintf(p_, sizeof p_, "model.%d", i);                           \
        b[i] = fm_new(WID(p_), (src)->h / 2, (src)->w / 2);               \
        if (st == ORC_OK) st = conv_named(m, p_, &b[i], (src), 2, 1, 1);  \
    } while (0)
#define OUTW(L) (findf(m, "%s.cv2.conv.weight", L) ? findf(m, "%s.cv2.conv.weight", L)->dims[0] : 0)
    DOWN(0, &x);
    emit(cb, user, "stage_01_buf0", &b[0]);
    DOWN(1, &b[0]);
    emit(cb, user, "stage_02_buf1", &b[1]);
    b[2] = fm_new(OUTW("model.2"), b[1].h, b[1].w);
    if (st == ORC_OK) st = c3k2_plain(m, "model.2", 1, 1, &b[2], &b[1]);
    emit(cb, user, "stage_03_buf2", &b[2]);
    DOWN(3, &b[2]);
    emit(cb, user, "stage_04_buf3", &b[3]);
    b[4] = fm_new(OUTW("model.4"), b[3].h, b[3].w);
    if (st == ORC_OK) st = c3k2_plain(m, "model.4", 1, 1, &b[4], &b[3]);
    emit(cb, user, "stage_05_buf4", &b[4]);
    DOWN(5, &b[4]);
    emit(cb, user, "stage_06_buf5", &b[5]);
    b[6] = fm_new(OUTW("model.6"), b[5].h, b[5].w);
    if (st == ORC_OK) st = c3k2_c3k(m, "model.6", &b[6], &b[5]);
    emit(cb, user, "stage_07_buf6", &b[6]);
    DOWN(7, &b[6]);
    emit(cb, user, "stage_08_buf7", &b[7]);
    b[8] = fm_new(OUTW("model.8"), b[7].h, b[7].w);
    if (st == ORC_OK) st = c3k2_c3k(m, "model.8", &b[8], &b[7]);
    emit(cb, user, "stage_09_buf8", &b[8]);
    b[9] = fm_new(OUTW("model.9"), b[8].h, b[8].w);
    if (st == ORC_OK) st = sppf(m, "model.9", 5, 3, 1, &b[9], &b[8]);
    emit(cb, user, "stage_10_buf9", &b[9]);
    b[10] = fm_new(OUTW("model.10"), b[9].h, b[9].w);
    if (st == ORC_OK) st = c2psa(m, "model.10", 1, 0.5f, 0.5f, &b[10], &b[9]);
    emit(cb, user, "stage_11_buf10", &b[10]);
    b[11] = upsample2(&b[10]);
    emit(cb, user, "stage_12_buf11", &b[11]);
    b[12] = concat2(&b[11], &b[6]);
    emit(cb, user, "stage_13_buf12", &b[12]);
    b[13] = fm_new(OUTW("model.13"), b[12].h, b[12].w);
    if (st == ORC_OK) st = c3k2_c3k(m, "model.13", &b[13], &b[12]);
    emit(cb, user, "stage_14_buf13", &b[13]);
    b[14] = upsample2(&b[13]);
    emit(cb, user, "stage_15_buf14", &b[14]);
    b[15] = concat2(&b[14], &b[4]);
    emit(cb, user, "stage_16_buf15", &b[15]);
    b[16] = fm_new(OUTW("model.16"), b[15].h, b[15].w);
    if (st == ORC_OK) st = c3k2_c3k(m, "model.16", &b[16], &b[15]);
    emit(cb, user, "stage_17_buf16", &b[16]);
    DOWN(17, &b[16]);
    emit(cb, user, "stage_18_buf17", &b[17]);
    b[18] = concat2(&b[17], &b[13]);
    emit(cb, user, "stage_19_buf18", &b[18]);
    b[19] = fm_new(OUTW("model.19"), b[18].h, b[18].w);
    if (st == ORC_OK) st = c3k2_c3k(m, "model.19", &b[19], &b[18]);
    emit(cb, user, "stage_20_buf19", &b[19]);
    DOWN(20, &b[19]);
    emit(cb, user, "stage_21_buf20", &b[20]);
    b[21] = concat2(&b[20], &b[10]);
    emit(cb, user, "stage_22_buf21", &b[21]);
    b[22] = fm_new(OUTW("model.22"), b[21].h, b[21].w);
    if (st == ORC_OK) st = c3k2_attn(m, "model.22", &b[22], &b[21]);
    emit(cb, user, "stage_23_buf22", &b[22]);
    if (st == ORC_OK) {
        const fmap* feats[3] = {&b[16], &b[19], &b[22]};
        st = detect(m, feats, max_det, dets, logits, boxes);
    }
    if (st == ORC_OK && cb) {
        cb(user, "stage_24_buf23", dets, 1, max_det, 6, 1);
        cb(user, "stage_25_detect", dets, 1, max_det, 6, 1);
    }
    for (int i = 0; i < 23; ++i) fm_free(&b[i]);
#undef WID
#undef DOWN
#undef OUTW
    return st;
}

/* ------------------------------------------------ block entry points (tests)
 * Each takes NCHW batch-1 data and weights already added under `prefix`. */
int orc_conv_block(void* h, const char* prefix, const float* in, int c, int hh, int ww, int stride, int pad, int act,
                   float* out) {
    orc_model* m = (orc_model*)h;
    orc_tensor* w = findf(m, "%s.conv.weight", prefix);
    orc_tensor* b = findf(m, "%s.conv.bias", prefix);
    if (!w) return ORC_ERR_MISSING;
    fmap x = {(float*)in, c, hh, ww};
    fmap y = {out, w->dims[0], (hh + 2 * pad - w->dims[2]) / stride + 1, (ww + 2 * pad - w->dims[3]) / stride + 1};
    conv(&y, &x, w, b, stride, pad, act);
    return ORC_OK;
}

int orc_c3k2(void* h, const char* prefix, int n, int shortcut, const float* in, int c, int hh, int ww, float* out,
             int co) {
    fmap x = {(float*)in, c, hh, ww}, y = {out, co, hh, ww};
    return c3k2_plain((orc_model*)h, prefix, n, shortcut, &y, &x);
}

int orc_c3k2_c3k(void* h, const char* prefix, const float* in, int c, int hh, int ww, float* out, int co) {
    fmap x = {(float*)in, c, hh, ww}, y = {out, co, hh, ww};
    return c3k2_c3k((orc_model*)h, prefix, &y, &x);
}

int orc_sppf(void* h, const char* prefix, int k, int n_pool, int shortcut, const float* in, int c, int hh, int ww,
             float* out, int co) {
    fmap x = {(float*)in, c, hh, ww}, y = {out, co, hh, ww};
    return sppf((orc_model*)h, prefix, k, n_pool, shortcut, &y, &x);
}

int orc_c2psa(void* h, const char* prefix, int n_blocks, const float* in, int c, int hh, int ww, float* out, int co) {
    fmap x = {(float*)in, c, hh, ww}, y = {out, co, hh, ww};
    return c2psa((orc_model*)h, prefix, n_blocks, 0.5f, 0.5f, &y, &x);
}

int orc_c3(void* h, const char* prefix, int shortcut, const float* in, int c, int hh, int ww, float* out, int co) {
    fmap x = {(float*)in, c, hh, ww}, y = {out, co, hh, ww};
    return c3((orc_model*)h, prefix, shortcut, &y, &x);
}

int orc_psablock(void* h, const char* prefix, const float* in, int c, int hh, int ww, int heads, float* out) {
    fmap x = {(float*)in, c, hh, ww}, y = {out, c, hh, ww};
    return psablock((orc_model*)h, prefix, heads, 0.5f, 1, &y, &x);
}

int orc_dwconv(void* h, const char* prefix, const float* in, int c, int hh, int ww, int act, float* out) {
    orc_model* m = (orc_model*)h;
    orc_tensor* w = findf(m, "%s.conv.weight", prefix);
    orc_tensor* b = findf(m, "%s.conv.bias", prefix);
    if (!w) return ORC_ERR_MISSING;
    fmap x = {(float*)in, c, hh, ww}, y = {out, c, hh, ww};
    dwconv(&y, &x, w, b, act);
    return ORC_OK;
}
