/*
 * ring.h - CPU->GPU CommandRing of 32-byte Descriptors.
 * Drop-in for reference include/ring.h:8-75 and src/ring.c:10-58:
 * same head/tail cache lines, 4,096 slots aligned to 128 B,
 * ring_acquire(n) -> masked position or UINT32_MAX, ring_commit(n),
 * ring_consume -> 1/0.
 *
 * The consumer of this ring on B200 is a single elected GPU thread (see
 * rlrt.h rt_decode_worker_launch), which keeps it strictly SPSC.
 */
#pragma once
#include <stddef.h>
#include <stdint.h>
#include "descriptor.h"
#include "completion.h"

typedef struct __attribute__((packed)) {
    __attribute__((aligned(64))) volatile uint32_t head;
    uint8_t pad[60];
} RingHead;

typedef struct __attribute__((packed)) {
    __attribute__((aligned(64))) volatile uint32_t tail;
    uint8_t pad[60];
} RingTail;

typedef struct {
    __attribute__((aligned(64))) RingHead cons;
    __attribute__((aligned(64))) RingTail prod;
    __attribute__((aligned(DESCRIPTOR_ALIGN))) Descriptor slots[RING_SIZE];
} CommandRing;

RT_STATIC_ASSERT(offsetof(CommandRing, prod) == 64, "CommandRing layout");
RT_STATIC_ASSERT(offsetof(CommandRing, slots) == 128, "CommandRing layout");

/* Producer: room for n more descriptors?  Returns the masked slot index of
 * the first one, or UINT32_MAX when fewer than n slots are free. */
static inline RT_HD uint32_t
ring_acquire(CommandRing *ring, uint32_t n)
{
    uint32_t head = rt_load_acquire_u32(&ring->cons.head);
    uint32_t tail = rt_load_relaxed_u32(&ring->prod.tail);
    if ((uint32_t)RING_SIZE - (tail - head) < n)
        return UINT32_MAX;
    return tail & (RING_SIZE - 1);
}

/* Producer: publish n descriptors written after ring_acquire. */
static inline RT_HD void
ring_commit(CommandRing *ring, uint32_t n)
{
    uint32_t tail = rt_load_relaxed_u32(&ring->prod.tail);
    rt_store_release_u32(&ring->prod.tail, tail + n);
}

/* Consumer: 1 when one descriptor was copied out, 0 when the ring is empty. */
static inline RT_HD int
ring_consume(CommandRing *ring, Descriptor *desc)
{
    uint32_t head = rt_load_relaxed_u32(&ring->cons.head);
    uint32_t tail = rt_load_acquire_u32(&ring->prod.tail);
    if (head == tail)
        return 0;
    rt_copy_bytes(desc, &ring->slots[head & (RING_SIZE - 1)], sizeof(Descriptor));
    rt_store_release_u32(&ring->cons.head, head + 1u);
    return 1;
}

#ifdef __cplusplus
extern "C" {
#endif
CommandRing *ring_create(void);
void ring_destroy(CommandRing *ring);
CompletionRing *comp_ring_create(void);
void comp_ring_destroy(CompletionRing *ring);
#ifdef __cplusplus
}
#endif
