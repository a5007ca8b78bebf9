/* ring.c - lifetime of the CommandRing, CompletionRing, RequestRing and
 * DoneRing (reference src/ring.c:10-58 and bench/bench_gpu_scheduler.cu:41-46).
 * All four live in pinned, device-mapped host memory so that the GPU worker
 * can be the other end of each ring. */
#include "ring.h"
#include "request.h"
#include "rt_hostmem.h"

CommandRing *
ring_create(void)
{
    return (CommandRing *)rt_host_alloc_shared(sizeof(CommandRing));
}

void
ring_destroy(CommandRing *ring)
{
    rt_host_free_shared(ring);
}

CompletionRing *
comp_ring_create(void)
{
    return (CompletionRing *)rt_host_alloc_shared(sizeof(CompletionRing));
}

void
comp_ring_destroy(CompletionRing *ring)
{
    rt_host_free_shared(ring);
}

RequestRing *
req_ring_create(void)
{
    return (RequestRing *)rt_host_alloc_shared(sizeof(RequestRing));
}

void
req_ring_destroy(RequestRing *r)
{
    rt_host_free_shared(r);
}

DoneRing *
done_ring_create(void)
{
    return (DoneRing *)rt_host_alloc_shared(sizeof(DoneRing));
}

void
done_ring_destroy(DoneRing *r)
{
    rt_host_free_shared(r);
}
