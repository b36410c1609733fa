/*
 * Harness around the reference implementation -- TEST INFRASTRUCTURE ONLY.
 *
 * Linked with the reference's own src/{tensor,utils,layers,detection,detect,
 * model}.c compiled from its sources by oracle/Makefile into
 * oracle/_ref/libyolo_ref.so.  It drives the reference through its public API
 * (model_create / model_load_weights / model_forward_ex, include/model.h) the
 * way tests/dump_model_stages.c does, with three additions the reference has
 * no entry point for:
 *   - any input size that is a multiple of 32 (model_create scales its buffers);
 *   - other widths: model_create sizes buffers for the n width, so for a width
 *     multiplier > 1 the public model_t.buffers are re-allocated wider;
 *   - pre-sigmoid class logits, recomputed from the stage buffers P3/P4/P5 with
 *     the reference's own layer functions and weights (detect.c:193-232).
 */
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

#include "detect.h"
#include "layers.h"
#include "model.h"
#include "tensor.h"
#include "utils.h"

static const int k_channels[23] = {16, 32, 64, 64, 128, 128, 128, 256, 256, 256, 256, 256,
                                   384, 128, 128, 256, 64, 64, 192, 128, 128, 384, 256};
static const int k_div[23] = {2, 4, 4, 8, 8, 16, 16, 32, 32, 32, 32, 16, 16, 16, 8, 8, 8, 16, 16, 16, 32, 32, 32};

static int widen(model_t* m, int H, int W, int mult) {
    if (mult == 1) return 0;
    for (int k = 0; k < 23; ++k) {
        tensor_free(&m->buffers[k]);
        if (tensor_allocate(&m->buffers[k], 1, k_channels[k] * mult, H / k_div[k], W / k_div[k]) != SUCCESS) return -1;
    }
    return 0;
}

static int cls_logits(model_t* m, float* logits) {
    const tensor_t* feats[3] = {&m->buffers[16], &m->buffers[19], &m->buffers[22]};
    const int nc = m->num_classes;
    const char* br = model_get_weight(m, "model.23.one2one_cv2.0.0.conv.weight") ? "one2one_cv3" : "cv3";
    int N = 0;
    for (int s = 0; s < 3; ++s) N += feats[s]->dims[2] * feats[s]->dims[3];
    int base = 0;
    char nm[200];
    for (int s = 0; s < 3; ++s) {
        const tensor_t* f = feats[s];
        const int h = f->dims[2], w = f->dims[3], hw = h * w;
#define W_(suffix) (snprintf(nm, sizeof nm, "model.23.%s.%d.%s", br, s, suffix), model_get_weight(m, nm))
        tensor_t* dw0 = W_("0.0.conv.weight");
        tensor_t* db0 = W_("0.0.conv.bias");
        tensor_t* pw0 = W_("0.1.conv.weight");
        tensor_t* pb0 = W_("0.1.conv.bias");
        tensor_t* dw1 = W_("1.0.conv.weight");
        tensor_t* db1 = W_("1.0.conv.bias");
        tensor_t* pw1 = W_("1.1.conv.weight");
        tensor_t* pb1 = W_("1.1.conv.bias");
        tensor_t* wf = W_("2.weight");
        tensor_t* bf = W_("2.bias");
#undef W_
        if (!dw0 || !db0 || !pw0 || !pb0 || !dw1 || !db1 || !pw1 || !pb1 || !wf || !bf) return -1;
        const int c3 = pw0->dims[0];
        tensor_t t0, t1, t2, t3, cls;
        tensor_allocate(&t0, 1, f->dims[1], h, w);
        tensor_allocate(&t1, 1, c3, h, w);
        tensor_allocate(&t2, 1, c3, h, w);
        tensor_allocate(&t3, 1, c3, h, w);
        tensor_allocate(&cls, 1, nc, h, w);
        conv_params_t p1 = {1, 0, 1};
        dwconv3x3_same_forward(&t0, f, dw0, db0);
        silu_forward(&t0);
        conv_block_forward(&t1, &t0, pw0, pb0, p1, true);
        dwconv3x3_same_forward(&t2, &t1, dw1, db1);
        silu_forward(&t2);
        conv_block_forward(&t3, &t2, pw1, pb1, p1, true);
        conv2d_forward(&cls, &t3, wf, bf, p1);
        for (int j = 0; j < hw; ++j)
            for (int c = 0; c < nc; ++c) logits[(size_t)(base + j) * nc + c] = cls.data[(size_t)c * hw + j];
        tensor_free(&t0);
        tensor_free(&t1);
        tensor_free(&t2);
        tensor_free(&t3);
        tensor_free(&cls);
        base += hw;
    }
    return 0;
}

/* One forward of one image [1,3,H,W]; dets receives [max_det, 6].
 * stage_path (nullable) receives the reference's stage dump.  logits
 * (nullable) receives [N, nc] anchor-major pre-sigmoid logits.  Returns the
 * reference's status, or -1 on a harness failure. */
int ref_forward(const char* weights, const float* in, int H, int W, int width_mult, int max_det, float* dets,
                const char* stage_path, float* logits) {
    model_t m;
    if (model_create(&m, W, H) != SUCCESS) return -1;
    if (widen(&m, H, W, width_mult) != 0) return -1;
    tensor_free(&m.buffers[23]);
    tensor_allocate(&m.buffers[23], 1, max_det, 6, 1);
    status_t st = model_load_weights(&m, weights);
    if (st != SUCCESS) {
        model_destroy(&m);
        return (int)st;
    }
    tensor_t x, out;
    x.data = (float*)in;
    x.dims[0] = 1;
    x.dims[1] = 3;
    x.dims[2] = H;
    x.dims[3] = W;
    x.stride[3] = 1;
    x.stride[2] = W;
    x.stride[1] = H * W;
    x.stride[0] = 3 * H * W;
    x.is_owner = false;
    tensor_allocate(&out, 1, max_det, 6, 1);
    FILE* f = stage_path ? fopen(stage_path, "wb") : NULL;
    st = model_forward_ex(&m, &x, &out, f, NULL);
    if (f) fclose(f);
    if (st == SUCCESS) {
        memcpy(dets, out.data, (size_t)max_det * 6 * sizeof(float));
        if (logits && cls_logits(&m, logits) != 0) st = (status_t)-1;
    }
    tensor_free(&out);
    model_destroy(&m);
    return (int)st;
}

/* C11 timespec_get: the reference headers are strict ISO C (their timer_t
 * clashes with POSIX), so clock_gettime is not declared here. */
static double now_s(void) {
    struct timespec ts;
    timespec_get(&ts, TIME_UTC);
    return (double)ts.tv_sec + 1e-9 * (double)ts.tv_nsec;
}

/* Loads once, then times `reps` forwards of the given image; returns the
 * total wall time in seconds (or a negative value on failure). */
double ref_time_forwards(const char* weights, const float* in, int H, int W, int width_mult, int reps) {
    model_t m;
    if (model_create(&m, W, H) != SUCCESS || widen(&m, H, W, width_mult) != 0) return -1.0;
    if (model_load_weights(&m, weights) != SUCCESS) return -2.0;
    tensor_t x, out;
    x.data = (float*)in;
    x.dims[0] = 1;
    x.dims[1] = 3;
    x.dims[2] = H;
    x.dims[3] = W;
    x.is_owner = false;
    tensor_allocate(&out, 1, 300, 6, 1);
    const double t0 = now_s();
    for (int r = 0; r < reps; ++r)
        if (model_forward(&m, &x, &out) != SUCCESS) return -3.0;
    const double t = now_s() - t0;
    tensor_free(&out);
    model_destroy(&m);
    return t;
}

/* A loaded reference model for repeated timed forwards (bench reference arm). */
typedef struct {
    model_t m;
    tensor_t out;
    int H, W;
} ref_handle;

void* ref_open(const char* weights, int H, int W, int width_mult) {
    ref_handle* h = (ref_handle*)calloc(1, sizeof(ref_handle));
    if (!h) return NULL;
    if (model_create(&h->m, W, H) != SUCCESS || widen(&h->m, H, W, width_mult) != 0 ||
        model_load_weights(&h->m, weights) != SUCCESS || tensor_allocate(&h->out, 1, 300, 6, 1) != SUCCESS) {
        free(h);
        return NULL;
    }
    h->H = H;
    h->W = W;
    return h;
}

/* One model_forward of image `in` [1,3,H,W]; dets (nullable) gets [300,6]. */
int ref_run(void* p, const float* in, float* dets) {
    ref_handle* h = (ref_handle*)p;
    tensor_t x;
    x.data = (float*)in;
    x.dims[0] = 1;
    x.dims[1] = 3;
    x.dims[2] = h->H;
    x.dims[3] = h->W;
    x.is_owner = false;
    status_t st = model_forward(&h->m, &x, &h->out);
    if (st == SUCCESS && dets) memcpy(dets, h->out.data, 300 * 6 * sizeof(float));
    return (int)st;
}

void ref_close(void* p) {
    ref_handle* h = (ref_handle*)p;
    if (!h) return;
    tensor_free(&h->out);
    model_destroy(&h->m);
    free(h);
}

/* Reference layer calls on raw arrays, for block-level comparisons. */
int ref_postprocess(const float* pred, int N, int nc, int max_det, int cap, float* out) {
    tensor_t o;
    if (tensor_allocate(&o, 1, cap, 6, 1) != SUCCESS) return -1;
    status_t st = detect_postprocess_from_pred(pred, N, nc, max_det, &o);
    memcpy(out, o.data, (size_t)cap * 6 * sizeof(float));
    tensor_free(&o);
    return (int)st;
}
