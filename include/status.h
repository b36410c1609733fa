#ifndef STATUS_H
#define STATUS_H

/* Status codes of the YOLO26 host API.
 *
 * The first seven values keep the numbering of the reference's status_t
 * (include/status.h:4-12 of phucb2/yolo-baremetal) so that callers compiled
 * against the reference header see identical codes.  The device backend adds
 * two codes at the end; existing values keep their ABI:
 *   ERROR_DEVICE  - a CUDA call failed, or a kernel reported an error flag
 *                   (for example a bounded barrier wait that gave up).
 *   ERROR_TIMEOUT - a host-side deadline on a GPU shard expired.
 */
typedef enum {
    SUCCESS = 0,
    ERROR_NULL_POINTER,
    ERROR_INVALID_DIMS,
    ERROR_OUT_OF_MEMORY,
    ERROR_NOT_IMPLEMENTED,
    ERROR_FILE_NOT_FOUND,
    ERROR_INVALID_FORMAT,
    ERROR_DEVICE,
    ERROR_TIMEOUT
} status_t;

#endif
