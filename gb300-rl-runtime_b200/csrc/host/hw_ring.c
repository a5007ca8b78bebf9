/* hw_ring.c - exported halves of the hw_desc_t ring (reference
 * src/hw_ring.c:6-42): system-scope acquire/release helpers and the ring
 * lifetime calls. */
#include "hw_ring.h"
#include "rt_hostmem.h"

#include <string.h>

uint32_t
hw_ring_load_acquire(volatile uint32_t *p)
{
    return rt_load_acquire_u32(p);
}

void
hw_ring_store_release(volatile uint32_t *p, uint32_t value)
{
    rt_store_release_u32(p, value);
}

hw_ring_t *
hw_ring_create(void)
{
    return (hw_ring_t *)rt_host_alloc_shared(sizeof(hw_ring_t));
}

void
hw_ring_reset(hw_ring_t *ring)
{
    if (ring)
        memset((void *)ring, 0, sizeof(*ring));
}

void
hw_ring_destroy(hw_ring_t *ring)
{
    rt_host_free_shared(ring);
}
