/* k3_gpu_internal.h -- shared by the C99 drop-in sources (not installed, not exported). */
#ifndef K3_GPU_INTERNAL_H
#define K3_GPU_INTERNAL_H

#include "k3cuda.h"

/* The process-wide libk3cuda context of the drop-ins (created on first use; aborts on
 * failure like every drop-in). */
__attribute__((visibility("hidden"))) k3cuda_ctx *k3g_ctx(void);

#endif
