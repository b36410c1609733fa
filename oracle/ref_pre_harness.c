/* Test infrastructure only: exposes the reference's image preprocessing,
 * which lives in static functions of src/main.c (resize_rgb_bilinear,
 * preprocess) and tests/dump_model_stages.c (load_rgb_resized), by compiling
 * those files unchanged from their own location (oracle/Makefile adds their
 * directories to the include path).  Their main() functions are renamed and
 * never called; stb_image is compiled static in each unit; the camera calls
 * main.c links against are stubs (the camera is a macOS device). */
#define STB_IMAGE_STATIC
#define main yb_ref_unused_app_main
#include "main.c"
#undef main

void ref_resize_rgb_bilinear(const uint8_t* src, int sw, int sh, uint8_t* dst, int dw, int dh) {
    resize_rgb_bilinear(src, sw, sh, dst, dw, dh);
}

void ref_preprocess(float* nchw, const uint8_t* rgb, int w, int h) {
    tensor_t t;
    memset(&t, 0, sizeof t);
    t.data = nchw;
    t.dims[0] = 1;
    t.dims[1] = 3;
    t.dims[2] = h;
    t.dims[3] = w;
    preprocess(&t, rgb, w, h);
}

status_t camera_create(camera_t** cam, int width, int height) {
    (void)cam;
    (void)width;
    (void)height;
    return ERROR_NOT_IMPLEMENTED;
}
status_t camera_destroy(camera_t* cam) {
    (void)cam;
    return ERROR_NOT_IMPLEMENTED;
}
status_t camera_start(camera_t* cam) {
    (void)cam;
    return ERROR_NOT_IMPLEMENTED;
}
status_t camera_stop(camera_t* cam) {
    (void)cam;
    return ERROR_NOT_IMPLEMENTED;
}
status_t camera_capture(camera_t* cam, uint8_t* buffer) {
    (void)cam;
    (void)buffer;
    return ERROR_NOT_IMPLEMENTED;
}
