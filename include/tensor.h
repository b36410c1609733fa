#ifndef TENSOR_H
#define TENSOR_H

/* Host tensor container of the YOLO26 API: NCHW float32, contiguous.
 * Same layout and function set as the reference's include/tensor.h:8-28
 * (phucb2/yolo-baremetal); the structure is the host ABI type that every
 * entry point of this library takes, so its fields and order are unchanged. */

#include <stdbool.h>
#include <stddef.h>
#include "status.h"

#ifdef __cplusplus
#define YB_RESTRICT __restrict
extern "C" {
#else
#define YB_RESTRICT restrict
#endif

typedef struct {
    float* YB_RESTRICT data;
    int dims[4];   /* N, C, H, W */
    int stride[4];
    bool is_owner;
} tensor_t;

status_t tensor_allocate(tensor_t* tensor, int n, int c, int h, int w);
status_t tensor_free(tensor_t* tensor);
status_t tensor_copy(tensor_t* dest, const tensor_t* src);
status_t tensor_fill(tensor_t* tensor, float value);

/* C = alpha * A * B + beta * C with A: M x K, B: K x N, C: M x N, all row-major
 * host arrays.  Runs on the GPU (tcgen05 split-bf16 GEMM). */
status_t tensor_gemm(float* C, const float* A, const float* B,
                     int M, int N, int K,
                     float alpha, float beta);

void* malloc_aligned(size_t size, size_t alignment);
void free_aligned(void* ptr);

#ifdef __cplusplus
}
#endif

#endif
