/*
 * hw_ring.h - SPSC ring of 64-byte hw_desc_t records.
 *
 * Drop-in for reference include/hw_ring.h:1-69 and src/hw_ring.c:6-42:
 * same 65,536-slot capacity, head and tail on their own cache lines,
 * free-running u32 indices, push/pop returning 0 on success and -1 when
 * full/empty.
 *
 * B200 difference: hw_ring_create() returns pinned, device-mapped host
 * memory (cudaHostAllocMapped) when a CUDA device is present, so the same
 * ring can be consumed by a GPU kernel; the device address equals the host
 * address under UVA.  Without a device it returns ordinary aligned memory.
 */
#pragma once
#include <stddef.h>
#include <stdint.h>
#include "hw_desc.h"

#define HW_RING_SIZE (1u << 16)
#define HW_RING_MASK (HW_RING_SIZE - 1u)

typedef struct {
    __attribute__((aligned(64))) volatile uint32_t head;  /* consumer-owned */
    char pad0[60];
    __attribute__((aligned(64))) volatile uint32_t tail;  /* producer-owned */
    char pad1[60];
    __attribute__((aligned(64))) hw_desc_t desc[HW_RING_SIZE];
} hw_ring_t;

RT_STATIC_ASSERT(offsetof(hw_ring_t, tail) == 64, "hw_ring_t layout");
RT_STATIC_ASSERT(offsetof(hw_ring_t, desc) == 128, "hw_ring_t layout");

#ifdef __cplusplus
extern "C" {
#endif
uint32_t hw_ring_load_acquire(volatile uint32_t *p);
void hw_ring_store_release(volatile uint32_t *p, uint32_t value);

hw_ring_t *hw_ring_create(void);
void hw_ring_reset(hw_ring_t *ring);
void hw_ring_destroy(hw_ring_t *ring);
#ifdef __cplusplus
}
#endif

static inline RT_HD int
hw_ring_full(hw_ring_t *ring)
{
    uint32_t h = rt_load_acquire_u32(&ring->head);
    uint32_t t = rt_load_acquire_u32(&ring->tail);
    return (t - h) >= HW_RING_SIZE;
}

static inline RT_HD int
hw_ring_empty(hw_ring_t *ring)
{
    uint32_t h = rt_load_acquire_u32(&ring->head);
    uint32_t t = rt_load_acquire_u32(&ring->tail);
    return h == t;
}

static inline RT_HD int
hw_ring_push(hw_ring_t *ring, const hw_desc_t *desc)
{
    uint32_t t = rt_load_acquire_u32(&ring->tail);
    uint32_t h = rt_load_acquire_u32(&ring->head);
    if ((t - h) >= HW_RING_SIZE)
        return -1;
    ring->desc[t & HW_RING_MASK] = *desc;
    rt_store_release_u32(&ring->tail, t + 1u);
    return 0;
}

static inline RT_HD int
hw_ring_pop(hw_ring_t *ring, hw_desc_t *out)
{
    uint32_t h = rt_load_acquire_u32(&ring->head);
    uint32_t t = rt_load_acquire_u32(&ring->tail);
    if (h == t)
        return -1;
    *out = ring->desc[h & HW_RING_MASK];
    rt_store_release_u32(&ring->head, h + 1u);
    return 0;
}
