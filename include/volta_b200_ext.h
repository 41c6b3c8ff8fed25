/*
 * Extensions of libvolta_cuda_backend.so that have no counterpart in the
 * reference seam.  They serve measurement only and never touch the RawStats
 * counters or any buffer: a caller of the reference ABI can ignore them.
 */
#ifndef VOLTA_B200_EXT_H
#define VOLTA_B200_EXT_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Record timing marker `slot` (0..7) on the context's stream. */
int volta_b200_timing_mark(void* ctx, int slot);
/* Wait for marker `end` and return the device time between two markers. */
int volta_b200_timing_elapsed(void* ctx, int start, int end, float* ms);
/* Kernels this context has launched since it was created. */
int volta_b200_launch_count(void* ctx, uint64_t* launches);

#ifdef __cplusplus
}
#endif
#endif /* VOLTA_B200_EXT_H */
