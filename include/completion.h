/*
 * completion.h - GPU->CPU completion ring of the per-step decode path.
 * Drop-in for reference include/completion.h:8-87: same 32-byte packed
 * Completion, same cache-line head/tail/overflow words, 4,096 slots,
 * push returns -1 and bumps `overflow` when full, poll returns 1/0.
 */
#pragma once
#include <stddef.h>
#include <stdint.h>
#include "rt_sync.h"

#define COMP_RING_SIZE 4096

#pragma pack(push, 1)
typedef struct {
    uint64_t seq_id;
    uint32_t token_id;
    uint32_t kv_block_offset;
    uint64_t reward_cookie;
    uint64_t cycles_taken;
} Completion;
#pragma pack(pop)

RT_STATIC_ASSERT(sizeof(Completion) == 32, "Completion must be 32 bytes");

typedef struct __attribute__((packed)) {
    __attribute__((aligned(64))) volatile uint32_t head;
    uint8_t pad[60];
} CompHead;

typedef struct __attribute__((packed)) {
    __attribute__((aligned(64))) volatile uint32_t tail;
    uint8_t pad[60];
} CompTail;

typedef struct __attribute__((packed)) {
    __attribute__((aligned(64))) volatile uint32_t value;
    uint8_t pad[60];
} CompCounter;

RT_STATIC_ASSERT(sizeof(CompHead) == 64, "CompHead is one cache line");
RT_STATIC_ASSERT(sizeof(CompTail) == 64, "CompTail is one cache line");
RT_STATIC_ASSERT(sizeof(CompCounter) == 64, "CompCounter is one cache line");

/* Status codes of the compact completion (see hw_desc.h completion_t). */
enum comp_status {
    COMP_STATUS_DONE          = 0x01,
    COMP_STATUS_REWARD_NEEDED = 0x02,
    COMP_STATUS_STOPPED       = 0xFF,
};

typedef struct {
    __attribute__((aligned(64))) CompHead cons;     /* CPU advances head */
    __attribute__((aligned(64))) CompTail prod;     /* GPU advances tail */
    __attribute__((aligned(64))) CompCounter overflow;
    __attribute__((aligned(128))) Completion slots[COMP_RING_SIZE];
} CompletionRing;

RT_STATIC_ASSERT(offsetof(CompletionRing, overflow) == 128, "CompletionRing layout");
RT_STATIC_ASSERT(offsetof(CompletionRing, slots) == 256, "CompletionRing layout");

static inline RT_HD void
comp_ring_record_overflow(volatile uint32_t *value)
{
    rt_count_u32(value);
}

/* Producer (GPU worker): 0 on success, -1 and overflow++ when full. */
static inline RT_HD int
comp_ring_push(CompletionRing *cr, const Completion *c)
{
    uint32_t head = rt_load_acquire_u32(&cr->cons.head);
    uint32_t tail = rt_load_relaxed_u32(&cr->prod.tail);
    if ((uint32_t)(tail - head) >= (uint32_t)COMP_RING_SIZE) {
        comp_ring_record_overflow(&cr->overflow.value);
        return -1;
    }
    cr->slots[tail & (COMP_RING_SIZE - 1)] = *c;
    rt_store_release_u32(&cr->prod.tail, tail + 1u);
    return 0;
}

/* Consumer (CPU): 1 when a completion was copied out, 0 when empty. */
static inline RT_HD int
comp_ring_poll(CompletionRing *cr, Completion *out)
{
    uint32_t head = rt_load_relaxed_u32(&cr->cons.head);
    uint32_t tail = rt_load_acquire_u32(&cr->prod.tail);
    if (head == tail)
        return 0;
    *out = cr->slots[head & (COMP_RING_SIZE - 1)];
    rt_store_release_u32(&cr->cons.head, head + 1u);
    return 1;
}
