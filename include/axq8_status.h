/* Status codes of the axion_b200 C ABI (include/axq8.h, include/axkv.h). */
#ifndef AXION_B200_AXQ8_STATUS_H
#define AXION_B200_AXQ8_STATUS_H

#define AXQ8_OK 0
#define AXQ8_ERR_INVALID (-1)      /* bad argument: null pointer, shape, alignment */
#define AXQ8_ERR_CUDA (-2)         /* a CUDA runtime call failed */
#define AXQ8_ERR_ALLOC (-3)        /* device or host allocation failed */
#define AXQ8_ERR_WAIT_TIMEOUT (-4) /* a bounded device-side wait gave up */
#define AXQ8_ERR_UNSUPPORTED (-5)  /* valid request outside the built kernels */
#define AXQ8_ERR_STATE (-6)        /* call out of order (e.g. decode before prefill) */

#endif
