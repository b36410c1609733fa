#ifndef UTILS_H
#define UTILS_H

/* Weight I/O, BatchNorm folding and timers of the YOLO26 host API
 * (reference: include/utils.h:43-54 of phucb2/yolo-baremetal).
 *
 * The reference names its timer struct `timer_t`, which collides with the
 * POSIX type of the same name whenever <time.h> exposes POSIX declarations
 * (any C++ or gnu11 translation unit).  This header names the struct
 * yb_timer_t; the layout (two uint64_t) and the function names are the same,
 * so objects built against either header link against this library.  Define
 * YB_LEGACY_TIMER_T before including it to also get the old spelling in
 * strict ISO C code. */

#include <stdint.h>
#include <stdio.h>
#include "status.h"
#include "tensor.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct {
    uint64_t start;
    uint64_t end;
} yb_timer_t;

#ifdef YB_LEGACY_TIMER_T
typedef yb_timer_t timer_t;
#endif

/* Monotonic wall-clock timers (nanosecond resolution on Linux). */
void timer_start(yb_timer_t* timer);
void timer_stop(yb_timer_t* timer);
double timer_elapsed_ms(const yb_timer_t* timer);

/* One record of the .bin layout: int32 name_len, name bytes (no NUL),
 * int32 ndim, int32 dims[ndim], float32 data[prod(dims)], little endian.
 * ndim <= 4; dims past ndim read as 1, so a rank-1 [C] record loads as
 * [C,1,1,1] and a rank-0 record is one element.  name must hold at least 128 bytes.  A truncated data block
 * returns ERROR_INVALID_FORMAT; end of file returns ERROR_FILE_NOT_FOUND. */
status_t load_named_tensor(FILE* f, char* name, tensor_t* tensor);
status_t save_named_tensor(FILE* f, const char* name, const tensor_t* tensor);

/* scale = gamma / sqrtf(var + 1e-5); W[c,:] *= scale; b = (b - mean)*scale + beta. */
void fold_bn(tensor_t* conv_w, tensor_t* conv_b,
             const tensor_t* bn_w, const tensor_t* bn_b,
             const tensor_t* bn_rm, const tensor_t* bn_rv);

#ifdef __cplusplus
}
#endif

#endif
