#define _POSIX_C_SOURCE 200112L
#include "rt_hostmem.h"

#include <stdlib.h>
#include <string.h>
#include <cuda_runtime_api.h>

static int
rt_have_device(void)
{
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) {
        (void)cudaGetLastError();
        return 0;
    }
    return n > 0;
}

void *
rt_host_alloc_shared(size_t bytes)
{
    void *p = NULL;
    if (rt_have_device()) {
        if (cudaHostAlloc(&p, bytes, cudaHostAllocMapped | cudaHostAllocPortable) == cudaSuccess) {
            memset(p, 0, bytes);
            return p;
        }
        (void)cudaGetLastError();
        p = NULL;
    }
    if (posix_memalign(&p, 4096, bytes) != 0)
        return NULL;
    memset(p, 0, bytes);
    return p;
}

int
rt_host_is_device_mapped(const void *p)
{
    unsigned int flags = 0;
    if (!p)
        return 0;
    if (cudaHostGetFlags(&flags, (void *)p) == cudaSuccess)
        return 1;
    (void)cudaGetLastError();
    return 0;
}

void
rt_host_free_shared(void *p)
{
    if (!p)
        return;
    if (rt_host_is_device_mapped(p))
        cudaFreeHost(p);
    else
        free(p);
}
