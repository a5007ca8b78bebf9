/*
 * rt_hostmem.h - host allocations shared with the GPU.
 *
 * Ring buffers are allocated pinned and device-mapped (cudaHostAllocMapped)
 * so that a persistent kernel can poll them; with UVA the device address is
 * the host address.  On a machine without a CUDA device the same call hands
 * out ordinary page-aligned memory, which is all a host-only producer and
 * consumer (e.g. hw_worker_sim) needs.
 */
#pragma once
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif
void *rt_host_alloc_shared(size_t bytes);  /* zero-filled, or NULL */
void rt_host_free_shared(void *p);
int rt_host_is_device_mapped(const void *p);
#ifdef __cplusplus
}
#endif
