#ifndef DETECTION_H
#define DETECTION_H

/* Detection list decode (reference: include/detection.h:1-24 of
 * phucb2/yolo-baremetal).  Host-side: filters at most max_det rows. */

#include "tensor.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct {
    float x1, y1, x2, y2;
    float score;
    int class_id;
} detection_t;

typedef struct {
    detection_t* detections;
    int count;
    int capacity;
} detection_results_t;

/* head_output: [1, max_det, >=6, >=1] rows x1,y1,x2,y2,score,class (pixels of
 * the model input).  Keeps rows with score > threshold, up to capacity. */
status_t decode_detections(detection_results_t* results, const tensor_t* head_output,
                           float threshold);

#ifdef __cplusplus
}
#endif

#endif
