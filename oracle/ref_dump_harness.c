/* Test infrastructure only: exposes load_rgb_resized, a static function of
 * the reference's tests/dump_model_stages.c (decode with stb_image, then the
 * pixel-centred bilinear resize), by compiling that file unchanged from its
 * own location.  Its main() is renamed and never called. */
#define STB_IMAGE_STATIC
#define main yb_ref_unused_dump_main
#include "dump_model_stages.c"
#undef main

uint8_t* ref_load_rgb_resized(const char* path, int out_w, int out_h) { return load_rgb_resized(path, out_w, out_h); }
void ref_free(void* p) { free(p); }
