#ifndef DETECT_H
#define DETECT_H

/* Detect head of YOLO26 (reference: include/detect.h:7-13 of
 * phucb2/yolo-baremetal).  reg_max = 1, end-to-end one-to-one branches. */

#include "model.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Runs the Detect head on host P3/P4/P5 feature maps ([1,C,H,W] each) with
 * the model's one2one_cv2/one2one_cv3 weights (cv2/cv3 when absent) and
 * writes the top-k rows into out_postprocess [1,max_det,6,1]. */
status_t detect_forward_one2one(model_t* model, int detect_module_idx,
                                const tensor_t* p3, const tensor_t* p4, const tensor_t* p5,
                                tensor_t* out_postprocess);

/* Top-k selection on host predictions: pred row-major (N, 4+nc) with xyxy
 * pixels followed by per-class sigmoid scores.  Writes min(max_det, N, cap)
 * rows [x1,y1,x2,y2,score,class] into out (1,cap,6,1) and zero-fills the
 * rest.  Order: score descending, ties by ascending anchor index (stage 1)
 * and ascending slot*nc+class (stage 2). */
status_t detect_postprocess_from_pred(const float* pred_n_4plusnc, int N, int nc, int max_det,
                                      tensor_t* out_postprocess);

#ifdef __cplusplus
}
#endif

#endif
