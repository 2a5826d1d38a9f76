// Status codes shared by the C ABI (return values) and the device status word.
#pragma once

// C-ABI return codes (0 = success).
#define PI05_OK 0
#define PI05_ERR_INVALID_ARG 1   /* null pointer or unsupported parameter value */
#define PI05_ERR_SHAPE 2         /* dimension not supported by the kernel (divisibility, limits) */
#define PI05_ERR_ALIGN 3         /* pointer or stride violates the 16-byte TMA / vector rule */
#define PI05_ERR_WORKSPACE 4     /* workspace missing or too small */
#define PI05_ERR_LAUNCH 5        /* cudaLaunch* failed (cudaGetLastError text via pi05_last_error) */
#define PI05_ERR_TMAP 6          /* cuTensorMapEncodeTiled rejected a tensor map */
#define PI05_ERR_DEVICE 7        /* the device status word reported an error (see bits below) */
#define PI05_ERR_DRIVER 8        /* driver entry point unavailable */

// Device status word bits (OR-ed by kernels into workspace word 0).
#define PI05_DEV_TIMEOUT_PRODUCER 0x1   /* TMA producer gave up waiting for a free stage */
#define PI05_DEV_TIMEOUT_MMA 0x2        /* MMA issuer gave up waiting for a loaded stage */
#define PI05_DEV_TIMEOUT_EPILOGUE 0x4   /* epilogue gave up waiting for the accumulator */
#define PI05_DEV_TIMEOUT_DRAIN 0x8      /* teardown gave up waiting for in-flight copies */
#define PI05_DEV_TIMEOUT_FLAG 0x10      /* a flag wait (test hook) ran out */
#define PI05_DEV_BAD_INDEX 0x20         /* an index input was out of range (row zero-filled) */
