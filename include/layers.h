#ifndef LAYERS_H
#define LAYERS_H

/* Layer-level entry points of the YOLO26 host API, one per reference layer
 * function (include/layers.h:12-77 of phucb2/yolo-baremetal), with the same
 * names, argument meaning and status codes.  Every call takes host NCHW
 * float32 tensors; this library stages them into HBM, runs the sm_100a
 * kernels (tcgen05 implicit-GEMM convolution with fused bias/SiLU/residual
 * epilogues, depthwise, pooling and attention kernels) and copies the result
 * back.  Scratch `buffers` arguments are accepted for signature compatibility;
 * the device path keeps its intermediates in HBM and leaves them untouched. */

#include "tensor.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct {
    int stride;
    int padding;
    int groups;
} conv_params_t;

/* Dense convolution (groups ignored, batch taken as 1 like the reference,
 * layers.c:41-81).  weight [co, ci, kh, kw]; bias [co] or NULL. */
status_t conv2d_forward(tensor_t* output, const tensor_t* input,
                        const tensor_t* weight, const tensor_t* bias,
                        conv_params_t params);

/* x / (1 + exp(-x)) in place (layers.c:10-21). */
status_t silu_forward(tensor_t* tensor);

/* Max pool, padding kernel/2 excluded from the max (layers.c:191-217). */
status_t pool2d_max_forward(tensor_t* output, const tensor_t* input, int kernel_size, int stride);

/* Nearest-neighbour upsample by an integer factor (layers.c:23-39). */
status_t upsample_nearest_forward(tensor_t* output, const tensor_t* input, int scale);

/* Channel concat; dim must be 1 (layers.c:219-228). */
status_t concat_forward(tensor_t* output, const tensor_t* input1, const tensor_t* input2, int dim);

/* conv2d then optional SiLU (layers.c:83-90). */
status_t conv_block_forward(tensor_t* output, const tensor_t* input,
                            const tensor_t* weight, const tensor_t* bias,
                            conv_params_t params, bool act);

/* cv1+SiLU, cv2+SiLU, + input when shortcut; padding (k-1)/2 (layers.c:92-108). */
status_t bottleneck_forward(tensor_t* output, const tensor_t* input,
                            const tensor_t* cv1_w, const tensor_t* cv1_b,
                            const tensor_t* cv2_w, const tensor_t* cv2_b,
                            bool shortcut, tensor_t* temp);

/* SPPF: cv1 1x1 without SiLU, n_pool chained stride-1 max pools, concat,
 * cv2 1x1 + SiLU, + input when shortcut and shapes match (layers.c:230-265). */
status_t sppf_forward(tensor_t* output, const tensor_t* input,
                      const tensor_t* cv1_w, const tensor_t* cv1_b,
                      const tensor_t* cv2_w, const tensor_t* cv2_b,
                      int kernel_size, int n_pool, bool shortcut,
                      tensor_t* buffers);

/* C3k2 (C2f path): cat(cv1 halves, n bottlenecks) -> cv2 (layers.c:110-154).
 * b_weights: n blocks of (cv1_w, cv1_b, cv2_w, cv2_b). */
status_t c3k2_forward(tensor_t* output, const tensor_t* input,
                      int n, bool shortcut,
                      const tensor_t* cv1_w, const tensor_t* cv1_b,
                      const tensor_t* cv2_w, const tensor_t* cv2_b,
                      const tensor_t* b_weights,
                      tensor_t* buffers);

/* C2PSA (layers.c:455-496).  psa_weights: n_blocks x 10 tensors
 * (qkv_w, qkv_b, proj_w, proj_b, pe_w, pe_b, ffn0_w, ffn0_b, ffn1_w, ffn1_b). */
status_t c2psa_forward(tensor_t* output, const tensor_t* input, int n_blocks, float e, float attn_ratio,
                       const tensor_t* cv1_w, const tensor_t* cv1_b, const tensor_t* cv2_w, const tensor_t* cv2_b,
                       const tensor_t* psa_weights, tensor_t* buffers);

/* One PSABlock: x1 = x + attn(x); out = x1 + ffn(x1) (layers.c:407-453). */
status_t psablock_forward(tensor_t* output, const tensor_t* input, bool shortcut,
                          const tensor_t* qkv_w, const tensor_t* qkv_b, const tensor_t* proj_w,
                          const tensor_t* proj_b, const tensor_t* pe_w, const tensor_t* pe_b,
                          const tensor_t* ffn0_w, const tensor_t* ffn0_b, const tensor_t* ffn1_w,
                          const tensor_t* ffn1_b, int num_heads, float attn_ratio);

/* Depthwise 3x3, padding 1, + bias; weight [C,1,3,3] (layers.c:269-290). */
status_t dwconv3x3_same_forward(tensor_t* out, const tensor_t* in, const tensor_t* w, const tensor_t* bias);

/* C3: cv3(cat(m(cv1(x)), cv2(x))) with ping-pong bottlenecks (layers.c:156-189). */
status_t c3_forward(tensor_t* output, const tensor_t* input, const tensor_t* cv1_w, const tensor_t* cv1_b,
                    const tensor_t* cv2_w, const tensor_t* cv2_b, const tensor_t* cv3_w, const tensor_t* cv3_b,
                    const tensor_t* b_weights, int n_bottles, bool shortcut, tensor_t* buffers);

#ifdef __cplusplus
}
#endif

#endif
