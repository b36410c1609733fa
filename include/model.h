#ifndef MODEL_H
#define MODEL_H

/* Model-level YOLO26 host API (reference: include/model.h:1-54 of
 * phucb2/yolo-baremetal).  The structures keep the reference's layout so a
 * caller of the reference links against this library unchanged; the device
 * replica (packed weights, HBM activations, captured CUDA graphs) is kept in
 * a side table keyed by the model_t pointer, so sizeof(model_t) is the same.
 *
 * Device selection: model_load_weights uploads to the CUDA device that is
 * current on the calling thread (cudaSetDevice), or to the device named by
 * the YB_DEVICE environment variable when it is set. */

#include <stdio.h>
#include "tensor.h"
#include "layers.h"
#include "detection.h"

#ifdef __cplusplus
extern "C" {
#endif

#define MAX_MODEL_LAYERS 32
/* Timed substeps of model_forward_ex, in the reference's order (model.c:680-706). */
#define MODEL_FORWARD_PROFILE_STEPS 25
/* Module index of the Detect head in the YOLO26 graph (model.23.*). */
#define YOLO26_DETECT_IDX 23

typedef struct {
    double ms_sum[MODEL_FORWARD_PROFILE_STEPS];
    double ms_last[MODEL_FORWARD_PROFILE_STEPS];
    unsigned runs;
} model_forward_profile_t;

void model_forward_profile_reset(model_forward_profile_t* p);
const char* model_forward_profile_step_name(int step_index);
void model_forward_profile_print_last(const model_forward_profile_t* p, FILE* fp, const char* title);
void model_forward_profile_print_aggregate(const model_forward_profile_t* p, FILE* fp);

typedef struct {
    char name[128];
    tensor_t tensor;
} named_tensor_t;

typedef struct {
    named_tensor_t* weights;
    int num_weights;

    tensor_t* buffers; /* host buffers; buffers[23] receives the detections */
    int num_buffers;

    int input_w, input_h;
    int num_classes;
} model_t;

status_t model_create(model_t* model, int input_w, int input_h);
status_t model_destroy(model_t* model);

/* One forward pass.  input: [B,3,H,W] float32 (B >= 1; the reference only
 * supports B = 1), output: [B,max_det,6,1] rows x1,y1,x2,y2,score,class. */
status_t model_forward(model_t* model, const tensor_t* input, tensor_t* output);

/* As model_forward.  stage_dump != NULL appends the 26 stage tensors
 * stage_00_input .. stage_25_detect in the reference's .bin record format
 * (NCHW float32; image 0 only when B > 1).  profile != NULL fills per-step
 * device times from CUDA events (the forward then runs eagerly, not from a
 * captured graph). */
status_t model_forward_ex(model_t* model, const tensor_t* input, tensor_t* output, FILE* stage_dump,
                          model_forward_profile_t* profile);

/* Additive batch entry: same as model_forward with B = input->dims[0]. */
status_t model_forward_batch(model_t* model, const tensor_t* input, tensor_t* output);

/* Reads the converter's .bin layout, folds BatchNorm exactly as the reference
 * (model.c:121-198, utils.c:81-106) and uploads the device replica. */
status_t model_load_weights(model_t* model, const char* path);
tensor_t* model_get_weight(model_t* model, const char* name);

#ifdef __cplusplus
}
#endif

#endif
