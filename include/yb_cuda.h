#ifndef YB_CUDA_H
#define YB_CUDA_H

/* C-ABI shim between the YOLO26 host API and the B200 (sm_100a) backend.
 *
 * Plain pointers and sizes only.  The reference has no device boundary; these
 * entry points replace the layer calls that src/model.c makes inside
 * model_forward_ex (model.c:764-903) and the Detect head call
 * detect_forward_one2one (detect.c:253-454) of phucb2/yolo-baremetal, so a
 * GPU-enabled model.c calls yb_cuda_forward where the reference walks its 24
 * layer steps.  One context = one device replica; contexts are independent
 * and may live on different GPUs (image-sharded multi-GPU needs no
 * collective: see yb_cuda_forward_sharded).
 *
 * All entry points return status_t (status.h).  CUDA failures map to
 * ERROR_OUT_OF_MEMORY (allocation) or ERROR_DEVICE (anything else, including a
 * kernel that reported a bounded-wait timeout); yb_cuda_last_error() returns a
 * one-line description of the last failure on the calling thread. */

#include "detection.h"
#include "model.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
    /* FP32 semantics: fp32 activations in HBM, convolutions as split-bf16
     * (hi+lo, three tcgen05 products) with fp32 accumulation in TMEM. */
    YB_PRECISION_FP32 = 0,
    /* INT8: int8 NHWC activations with per-tensor scales, int8 weights with
     * per-output-channel scales, convolutions on tcgen05 kind::i8 with int32
     * accumulation in TMEM and round-half-even requantisation (yb_int8.h
     * gives the per-layer rules); Detect's last convolutions dequantise to
     * fp32 for the decode and top-k. */
    YB_PRECISION_INT8 = 1
} yb_precision;

/* Scale table of an INT8 model: one positive float per named tensor.  A
 * convolution with weight prefix P writes tensor "P" (after its residual) and,
 * with SiLU, has the pre-activation scale "P:pre"; further "input" (the
 * network input), "<psa>.attn.ope" (attention output plus positional term)
 * for every attention block, and the Detect head's depthwise convolutions
 * (their own prefixes, with ":pre").  The CPU oracle's calibration produces
 * such a table from sample images (max |x| / 127 per tensor). */
typedef struct {
    const char* const* names;
    const float* scales;
    int n;
} yb_int8_scales;

/* Resize rule of the device preprocess (yb_cuda_forward_rgb8,
 * yb_cuda_preprocess_rgb8), both the reference's, bit for bit. */
typedef enum {
    /* src/main.c:18-51 resize_rgb_bilinear (image and camera paths): corners
     * aligned, source coordinate dx * (sw - 1) / (dw - 1), rounded half up. */
    YB_RESIZE_ALIGN_CORNERS = 0,
    /* tests/dump_model_stages.c:58-96 load_rgb_resized: pixel centres,
     * source coordinate (x + 0.5) * sw / dw - 0.5, truncated. */
    YB_RESIZE_HALF_PIXEL = 1
} yb_resize_mode;

/* Stage callback: called once per stage tensor (NCHW float32 host data of
 * image 0) with the reference's stage names stage_00_input .. stage_25_detect. */
typedef void (*yb_stage_cb)(void* user, const char* name, const float* nchw, int n, int c, int h, int w);

/* Creates a context on CUDA device `device` (its own stream and arena). */
status_t yb_cuda_init(int device, void** ctx);

/* Packs and uploads the BN-folded weights of `m` (after model_load_weights /
 * fold_all_bn).  YB_PRECISION_FP32: qparams must be NULL.  YB_PRECISION_INT8:
 * qparams is a const yb_int8_scales* (as for yb_cuda_set_int8). */
status_t yb_cuda_upload_weights(void* ctx, const model_t* m, yb_precision p, const void* qparams);

/* Switches the context's precision: n > 0 makes every later forward INT8
 * under this scale table (names[i] -> scales[i]; the weights are quantised
 * when a plan is first built), n = 0 returns to FP32.  Plans are rebuilt on
 * the next forward.  A scale the graph needs but the table lacks is reported
 * then, as ERROR_INVALID_DIMS naming the tensor. */
status_t yb_cuda_set_int8(void* ctx, const char* const* names, const float* scales, int n);

/* Fused block kernels (on by default): each Bottleneck of the C3k2 / C3k
 * blocks whose two 3x3 convolutions map C -> C channels with C = 16 or 32
 * runs as one launch, its intermediate kept in shared memory.  enable = 0
 * launches every convolution separately.  Results are bit-identical either
 * way; plans are rebuilt on the next forward. */
status_t yb_cuda_set_fusion(void* ctx, int enable);

/* INT8 calibration on the device: FP32 forwards of n images [n,3,H,W]
 * (host, float32; H, W multiples of 32) recording max |x| of every tensor the
 * INT8 plan names (conv outputs after their residual, SiLU pre-activations,
 * attention outputs, the input), giving scale = max|x| / 127 (1 for an
 * all-zero tensor), the rule of the CPU oracle's calibration.  The table is
 * kept in the context (yb_cuda_int8_scale_entry reads it, in name order);
 * apply != 0 also switches the context to INT8 under it, as
 * yb_cuda_set_int8 would.  *n_scales (nullable) receives its size. */
status_t yb_cuda_calibrate_int8(void* ctx, const float* images, int n, int H, int W, int apply, int* n_scales);

/* Entry i of the last calibration's table: name (NUL-terminated, cap bytes
 * available; ERROR_INVALID_DIMS when too small) and scale; either nullable. */
status_t yb_cuda_int8_scale_entry(void* ctx, int i, char* name, int cap, float* scale);

/* Stage tensor `idx` (0..22: the reference's stage_01_buf0 .. stage_23_buf22)
 * of image `image` of the last INT8 forward (not a pipelined one): out_nchw
 * [c][h][w] int8 (nullable) and its per-channel scales [c] (nullable; the
 * dequantised value is q * scales[channel]).  *c, *h, *w receive the shape. */
status_t yb_cuda_get_int8_stage(void* ctx, int idx, int image, signed char* out_nchw, float* scales, int* c, int* h,
                                int* w);

/* Convenience for hosts without a model_t: reads a converter-layout .bin,
 * folds BatchNorm like model_load_weights and uploads. */
status_t yb_cuda_load_bin(void* ctx, const char* path);

/* Device-side weight preparation.  yb_cuda_load_bin_device takes the same
 * converter .bin (converter.py:116-131) but folds BatchNorm on the GPU
 * (the rule of utils.c:81-106 / model.c:121-180, explicitly rounded, so the
 * folded values equal the host fold bit for bit); every later packing of
 * the weights (FP32 tcgen05 operand images, INT8 quantisation and layouts)
 * then also runs as GPU kernels.  The host reads the file and keeps only
 * names and shapes.
 *
 * yb_cuda_save_prepared writes a prepared-weight blob: the folded weights
 * and the packed FP32 operand image of every convolution.
 * yb_cuda_load_prepared restores a context from such a blob with one copy
 * of the folded weights and one of each packed image, without folding or
 * packing (fast start).  ERROR_INVALID_FORMAT for a file that is not a blob
 * of this version.
 *
 * yb_cuda_weight_image copies one prepared weight image to host memory:
 * kind 0 the folded fp32 tensor `name`; kind 1 the packed FP32 operand image
 * of convolution prefix `name` (e.g. "model.2.cv1") in n_tile-wide N tiles
 * (0 = the full tiling, else 64 or 128); kind 2 the packed INT8 operand image
 * of convolution prefix `name` in the last INT8 plan built.  *bytes receives
 * the size; out may be NULL to query it.  Either preparation path (host or
 * device) answers, so the two can be compared. */
status_t yb_cuda_load_bin_device(void* ctx, const char* path);
status_t yb_cuda_save_prepared(void* ctx, const char* path);
status_t yb_cuda_load_prepared(void* ctx, const char* path);
status_t yb_cuda_weight_image(void* ctx, const char* name, int kind, int n_tile, void* out, size_t cap,
                              size_t* bytes);

/* Forward on host buffers: in_nchw [B,3,H,W] float32 (H, W multiples of 32),
 * out_dets [B,max_det,6] float32.  The input is copied to HBM, the captured
 * graph for (B,H,W) runs, and the detections come back; the call returns
 * when they are in out_dets.  dump (nullable) receives the stage tensors;
 * step_ms (nullable, MODEL_FORWARD_PROFILE_STEPS doubles) receives per-step
 * device times.  Either one makes the forward run eagerly instead of from the
 * captured graph.  Without them, a batch of B >= 32 images with B a multiple
 * of 16 is pipelined: 16-image sub-batches rotate over three captured
 * graphs, each on its own stream, so that the input copies run back to back
 * and each sub-batch's graph overlaps the copies and graphs after it (use
 * pinned host buffers for the overlap to happen); the head tensors of such a
 * forward are not kept (yb_cuda_get_head). */
status_t yb_cuda_forward(void* ctx, const float* in_nchw, int B, int H, int W,
                         float* out_dets, int max_det,
                         yb_stage_cb dump, void* user, double* step_ms);

/* Forward from 8-bit images: rgb_hwc [B, src_h, src_w, 3] uint8 RGB (host,
 * pinned for full copy speed) is copied to the GPU (a quarter of the fp32
 * input's bytes), resized to H x W by `resize` (yb_resize_mode), scaled by
 * 1/255 into the plan's fp32 NCHW input (main.c:53-64) on the device, and
 * run; out_dets [B, max_det, 6] as yb_cuda_forward.  The network input equals
 * the reference's preprocess of the same pixels bit for bit.  The head
 * tensors are kept (yb_cuda_get_head). */
status_t yb_cuda_forward_rgb8(void* ctx, const unsigned char* rgb_hwc, int B, int src_h, int src_w, int resize,
                              int H, int W, float* out_dets, int max_det);

/* Streaming forward for a sequence of batches: queues the input copy, the
 * forward and the detections' copy of one batch and returns without waiting;
 * *ticket identifies the batch.  Two batches can be in flight per context
 * (two captured graphs on their own streams): the input copy of one runs while
 * the other computes.  A submit while both slots are busy first waits for the
 * older batch of the slot it reuses.  in_nchw and out_dets (pinned host memory
 * for the copies to overlap) must stay valid until yb_cuda_forward_wait
 * returns for the ticket; detections and errors are those of yb_cuda_forward.
 * The rgb8 form takes uint8 frames as yb_cuda_forward_rgb8 (the device
 * preprocess runs on the batch's stream).  Replacing weights or the precision
 * first finishes the batches in flight. */
status_t yb_cuda_forward_submit(void* ctx, const float* in_nchw, int B, int H, int W, float* out_dets, int max_det,
                                long long* ticket);
status_t yb_cuda_forward_rgb8_submit(void* ctx, const unsigned char* rgb_hwc, int B, int src_h, int src_w,
                                     int resize, int H, int W, float* out_dets, int max_det, long long* ticket);
/* Waits until the batch of `ticket` is complete (its detections are in its
 * out_dets).  A ticket that already completed returns SUCCESS. */
status_t yb_cuda_forward_wait(void* ctx, long long ticket);

/* The device preprocess alone: d_rgb [B, src_h, src_w, 3] uint8 and d_nchw
 * [B, 3, H, W] fp32 in the current device's memory; enqueued on `stream`
 * (NULL = the default stream), does not synchronize. */
status_t yb_cuda_preprocess_rgb8(const unsigned char* d_rgb, int B, int src_h, int src_w, int resize, float* d_nchw,
                                 int H, int W, void* stream);

/* Detection lists of the last forward (not a pipelined one): for each image,
 * decode_detections (detection.c:3-34) on the device -- the rows whose score
 * is not <= threshold, in row order, at most `capacity` -- then copied out:
 * out [B][capacity] detection_t, counts [B].  A compact alternative to
 * reading the [B, max_det, 6] rows. */
status_t yb_cuda_get_detections(void* ctx, float threshold, int capacity, detection_t* out, int* counts);

/* The same on device buffers: d_dets [B, rows, 6] fp32, d_out [B][capacity]
 * detection_t, d_counts [B]; enqueued on `stream` (NULL = the default
 * stream), does not synchronize. */
status_t yb_cuda_detections(const float* d_dets, int B, int rows, float threshold, int capacity, detection_t* d_out,
                            int* d_counts, void* stream);

/* Forward on device buffers already in this context's GPU memory:
 * d_in [B,3,H,W], d_out [B,max_det,6].  Enqueued on `stream` (a
 * cudaStream_t; NULL = the context's own stream); does not synchronize. */
status_t yb_cuda_forward_device(void* ctx, const float* d_in, int B, int H, int W,
                                float* d_out, int max_det, void* stream);

/* The HBM input [B,3,H,W] and output [B,max_det,6] buffers of the plan for
 * (B,H,W,max_det), creating the plan if needed.  Writing the input there and
 * calling yb_cuda_forward_device with the same pointers runs the captured
 * graph with no extra device copies. */
status_t yb_cuda_plan_io(void* ctx, int B, int H, int W, int max_det, float** d_in, float** d_out);

/* Copies the head tensors of the last forward, image-major (not available
 * after a pipelined yb_cuda_forward: ERROR_INVALID_DIMS):
 * logits [B,N,nc] (pre-sigmoid class logits) and boxes [B,N,4] (xyxy pixels),
 * N = anchors per image.  Either pointer may be NULL.  *n_anchors and *nc
 * receive N and nc when non-NULL. */
status_t yb_cuda_get_head(void* ctx, float* logits, float* boxes, int* n_anchors, int* nc);

/* Detect-head top-k on head tensors already in GPU memory, allocating
 * nothing.  No counterpart in the reference (its top-k,
 * detect_postprocess_from_pred, works on host memory).  For callers that
 * cannot allocate device memory: a serving process whose GPU memory is all
 * owned by its own pool allocator, or a per-frame loop that cannot take the
 * stall of cudaMalloc/cudaFree (cudaFree waits for all work on the device).
 *
 * d_logits [B,N,nc] pre-sigmoid class logits and d_boxes [B,N,4] xyxy, as
 * yb_cuda_get_head returns them; d_dets [B,max_det,6] receives
 * [x1,y1,x2,y2,score,class] rows in the order of yb_cuda_forward's output,
 * rows beyond min(max_det, N) zero-filled.  All three on the current device.
 * Enqueued on `stream` (a cudaStream_t; NULL = the default stream); does not
 * synchronize.
 *
 * Scratch (the per-anchor best scores) lives in one fixed array of 2^20
 * floats (4 MiB) inside the library's device code: B*N above 1048576
 * anchors, or min(max_det, N) above 1024, returns ERROR_INVALID_DIMS before
 * any launch.  Under CUDA's lazy module loading (the default since CUDA
 * 12.2) the array and the kernels are placed on a device when the library's
 * device code is first used there; from then on the device holds them until
 * the process exits.  yb_cuda_init does that loading for its device.  A
 * caller that never creates a context on a device should make one warm-up
 * call there before its pool allocator reserves the device's memory, and
 * before any stream capture (the first call on a device also looks the
 * array's address up, with that device current).  The cached address does
 * not survive cudaDeviceReset.  All calls on a device share the array, so
 * calls that overlap in time (other streams, other threads) race: order them
 * on one stream or with events. */
status_t yb_cuda_detect_topk_noalloc(const float* d_logits, const float* d_boxes, int B, int N, int nc,
                                     int max_det, float* d_dets, void* stream);

/* Image-sharded forward over G contexts (one per GPU): image range
 * [g*B/G, (g+1)*B/G) runs on ctxs[g] from its own host thread; results land
 * at the matching rows of out_dets.  Each shard is waited on with a host
 * deadline of timeout_ms (<= 0: no deadline); an expired deadline returns
 * ERROR_TIMEOUT after the other shards have finished or timed out.  After
 * ERROR_TIMEOUT the input copy of a late shard may still be queued on its
 * GPU: keep in_nchw valid until the next call on those contexts returns, or
 * until they are destroyed. */
status_t yb_cuda_forward_sharded(void* const* ctxs, int G, const float* in_nchw, int B, int H, int W,
                                 float* out_dets, int max_det, int timeout_ms);

/* One FP32 convolution on tensors already in GPU memory: conv2d_forward +
 * bias + optional SiLU (layers.c:41-90), with the kernel and operand mode
 * the model graph picks for the same shape.  Additive (the reference's
 * conv2d_forward takes host tensors and runs one image); used for the
 * isolated convolution sweep and its tests.
 *
 * yb_conv_create: w [co][ci][kh][kw] fp32 (BatchNorm already folded), b [co]
 * or NULL, kh = kw in {1, 3}, act 0 (none) or 1 (SiLU); packs and uploads to
 * `device`.  yb_conv_ci_pad returns the channel stride the input must have
 * (ci rounded up to a multiple of 8, extra channels zero), or 0 when the
 * handle reads an NCHW fp32 input [B,ci,H,W] (3x3 stride-2 convolutions of
 * <= 4 input channels with SiLU and 16/32/64 outputs: the first layer's
 * kernel).  Otherwise d_x is split NHWC: a bf16 plane hi [B,H,W,ci_pad]
 * followed by a bf16 plane lo of the same size, value = hi + lo.  d_y is
 * split NHWC [B,Ho,Wo,co8] (co rounded up to 8) the same way.  16-byte
 * aligned buffers.  Enqueued on `stream` (NULL = default stream); does not
 * synchronize.  yb_conv_check synchronizes and reads the handle's device
 * error word (bounded waits that gave up). */
status_t yb_conv_create(int device, const float* w, const float* b, int co, int ci, int kh, int kw, int stride,
                        int pad, int act, void** conv);
int yb_conv_ci_pad(void* conv);
status_t yb_conv_run(void* conv, const void* d_x, int B, int H, int W, void* d_y, void* stream);
status_t yb_conv_check(void* conv);
status_t yb_conv_destroy(void* conv);

/* Test hook of the kernel's bounded waits (no GPU fault involved): the next
 * yb_conv_run of this handle launches with its producer warps arming no
 * barrier and issuing no copy, and with a 1 ms bound on every wait.  The
 * UMMA issuer's first wait runs out; the kernel records the error, drains,
 * frees its tensor memory and returns, so yb_conv_check reports
 * ERROR_DEVICE and later runs are unaffected.  ERROR_NOT_IMPLEMENTED for the
 * first-layer (NCHW input) kernel, which has no barrier waits. */
status_t yb_conv_debug_withhold(void* conv);

/* One kernel launch of a plan, as measured by yb_cuda_profile_ops. */
typedef struct {
    int kind;     /* 0 tcgen05 conv, 1 stem conv, 2 depthwise, 3 max pool, 4 attention, 5 decode, 6 top-k */
    int step;     /* model_forward_profile_t step index */
    double ms;    /* mean device time of the launch */
    double flops; /* algorithmic FLOPs (2 x MACs) */
    double bytes; /* algorithmic HBM bytes: inputs and weights read once, outputs written once */
} yb_op_stat;

/* Runs the plan for (B,H,W,max_det) eagerly `reps` times with an event pair
 * around every launch.  *n_ops receives the number of launches in one
 * forward; stats (nullable, capacity cap) receives one record per launch. */
status_t yb_cuda_profile_ops(void* ctx, int B, int H, int W, int max_det, int reps, yb_op_stat* stats, int cap,
                             int* n_ops);

/* Host-side fault injection for deadline tests: the context's next sharded
 * calls sleep `ms` milliseconds on the host before enqueueing any GPU work
 * (0 disables).  No GPU work is stalled or faulted. */
status_t yb_cuda_debug_inject_stall(void* ctx, int ms);

/* Releases the context's device memory, graphs and stream. */
status_t yb_cuda_destroy(void* ctx);

/* Last failure on the calling thread ("" when none). */
const char* yb_cuda_last_error(void);

#ifdef __cplusplus
}
#endif

#endif
