/*
 * request.h - rollout admission (RequestRing, CPU->GPU), rollout completion
 * (DoneRing, GPU->CPU) and the GPU rollout slot table.
 *
 * Drop-in for reference include/request.h:12-150: the 34-byte packed
 * RolloutRequest, the 24-byte RolloutDone, 1,024-slot rings whose record
 * arrays start 128-byte aligned, the 256-slot GpuRolloutSlot table with its
 * free bitmap, and the same return conventions (acquire -> position or
 * UINT32_MAX, consume/pop -> 1/0, done push -> 0 or -1 with overflow++).
 *
 * request_id == UINT64_MAX is the worker stop sentinel.  The slot table
 * keeps only the low 32 bits of request_id (reference cu/gpu_scheduler.cu:44),
 * so the upper 32 bits never reach the done stream; this runtime uses them
 * as a routing field: bits 32..63 = shared-prefix id + 1 (0 = no prefix),
 * see RT_REQUEST_PREFIX().
 */
#pragma once
#include <stddef.h>
#include <stdint.h>
#include "rt_sync.h"

#define REQUEST_RING_SIZE 1024
#define GPU_MAX_ROLLOUTS 256

#pragma pack(push, 1)
typedef struct {
    uint64_t request_id;
    uint32_t max_tokens;
    uint32_t kv_blocks;
    float    temperature;
    uint16_t top_k;
    float    top_p;
    uint64_t rng_seed;
} RolloutRequest;

typedef struct {
    uint64_t request_id;
    uint32_t rollout_id;       /* slot index that ran the rollout */
    uint32_t tokens_generated;
    float    reward;
    uint32_t status;
} RolloutDone;
#pragma pack(pop)

RT_STATIC_ASSERT(sizeof(RolloutRequest) == 34, "RolloutRequest must be 34 bytes");
RT_STATIC_ASSERT(sizeof(RolloutDone) == 24, "RolloutDone must be 24 bytes");
RT_STATIC_ASSERT(offsetof(RolloutRequest, top_p) == 22, "RolloutRequest layout");
RT_STATIC_ASSERT(offsetof(RolloutRequest, rng_seed) == 26, "RolloutRequest layout");

#define RT_REQUEST_SENTINEL   UINT64_MAX
/* Shared-prefix routing field carried in request_id bits 32..63. */
#define RT_REQUEST_PREFIX(id) ((uint32_t)((uint64_t)(id) >> 32))
#define RT_REQUEST_ID(lo, prefix_plus_one) \
    (((uint64_t)(prefix_plus_one) << 32) | (uint64_t)(uint32_t)(lo))

typedef struct __attribute__((packed)) {
    __attribute__((aligned(64))) volatile uint32_t head;
    uint8_t pad[60];
} ReqHead;

typedef struct __attribute__((packed)) {
    __attribute__((aligned(64))) volatile uint32_t tail;
    uint8_t pad[60];
} ReqTail;

typedef struct __attribute__((packed)) {
    __attribute__((aligned(64))) volatile uint32_t value;
    uint8_t pad[60];
} ReqCounter;

typedef struct {
    __attribute__((aligned(64))) ReqHead cons;
    __attribute__((aligned(64))) ReqTail prod;
    __attribute__((aligned(128))) RolloutRequest slots[REQUEST_RING_SIZE];
} RequestRing;

typedef struct {
    __attribute__((aligned(64))) ReqHead cons;
    __attribute__((aligned(64))) ReqTail prod;
    __attribute__((aligned(64))) ReqCounter overflow;
    __attribute__((aligned(128))) RolloutDone slots[REQUEST_RING_SIZE];
} DoneRing;

RT_STATIC_ASSERT(offsetof(RequestRing, slots) == 128, "RequestRing layout");
RT_STATIC_ASSERT(offsetof(DoneRing, slots) == 256, "DoneRing layout");

typedef struct {
    uint32_t active;
    uint32_t request_id;        /* low 32 bits of RolloutRequest.request_id */
    uint32_t tokens_generated;
    uint32_t max_tokens;
    uint32_t kv_blocks;
    uint64_t rng_state[4];
    float    temperature;
    uint16_t top_k;
    float    top_p;
} GpuRolloutSlot;

typedef struct {
    GpuRolloutSlot slots[GPU_MAX_ROLLOUTS];
    uint64_t       bitmap[(GPU_MAX_ROLLOUTS + 63) / 64];  /* 1 = slot in use */
} GpuRolloutState;

RT_STATIC_ASSERT(sizeof(GpuRolloutSlot) == 72, "GpuRolloutSlot natural layout");
RT_STATIC_ASSERT(offsetof(GpuRolloutSlot, rng_state) == 24, "GpuRolloutSlot layout");
RT_STATIC_ASSERT(offsetof(GpuRolloutSlot, top_p) == 64, "GpuRolloutSlot layout");
RT_STATIC_ASSERT(sizeof(GpuRolloutState) == 72 * 256 + 32, "GpuRolloutState layout");

/* Producer (CPU): masked position of the next free request slot, or
 * UINT32_MAX when the ring is full. */
static inline RT_HD uint32_t
req_ring_acquire(RequestRing *r)
{
    uint32_t head = rt_load_acquire_u32(&r->cons.head);
    uint32_t tail = rt_load_relaxed_u32(&r->prod.tail);
    if ((uint32_t)REQUEST_RING_SIZE - (tail - head) < 1u)
        return UINT32_MAX;
    return tail & (REQUEST_RING_SIZE - 1);
}

/* Producer (CPU): publish the request written at the acquired position. */
static inline RT_HD void
req_ring_commit(RequestRing *r)
{
    uint32_t tail = rt_load_relaxed_u32(&r->prod.tail);
    rt_store_release_u32(&r->prod.tail, tail + 1u);
}

static inline RT_HD void
done_ring_record_overflow(volatile uint32_t *value)
{
    rt_count_u32(value);
}

/* Consumer (GPU): 1 when a request was copied out, 0 when empty. */
static inline RT_HD int
req_ring_consume(RequestRing *r, RolloutRequest *out)
{
    uint32_t head = rt_load_relaxed_u32(&r->cons.head);
    uint32_t tail = rt_load_acquire_u32(&r->prod.tail);
    if (head == tail)
        return 0;
    rt_copy_bytes(out, &r->slots[head & (REQUEST_RING_SIZE - 1)], sizeof(RolloutRequest));
    rt_store_release_u32(&r->cons.head, head + 1u);
    return 1;
}

/* Producer (GPU): 0 on success, -1 and overflow++ when the ring is full. */
static inline RT_HD int
done_ring_push(DoneRing *r, const RolloutDone *d)
{
    uint32_t head = rt_load_acquire_u32(&r->cons.head);
    uint32_t tail = rt_load_relaxed_u32(&r->prod.tail);
    if ((uint32_t)REQUEST_RING_SIZE - (tail - head) < 1u) {
        done_ring_record_overflow(&r->overflow.value);
        return -1;
    }
    RolloutDone *slot = &r->slots[tail & (REQUEST_RING_SIZE - 1)];
    rt_copy_bytes(slot, d, sizeof(RolloutDone));
    rt_store_release_u32(&r->prod.tail, tail + 1u);
    return 0;
}

/* Consumer (CPU): 1 when a done record was copied out, 0 when empty. */
static inline RT_HD int
done_ring_pop(DoneRing *r, RolloutDone *out)
{
    uint32_t head = rt_load_relaxed_u32(&r->cons.head);
    uint32_t tail = rt_load_acquire_u32(&r->prod.tail);
    if (head == tail)
        return 0;
    rt_copy_bytes(out, &r->slots[head & (REQUEST_RING_SIZE - 1)], sizeof(RolloutDone));
    rt_store_release_u32(&r->cons.head, head + 1u);
    return 1;
}

#ifdef __cplusplus
extern "C" {
#endif
/* Mapped-pinned allocation of the two rings (the reference allocates them
 * with cudaHostAlloc in its drivers, bench/bench_gpu_scheduler.cu:41-46). */
RequestRing *req_ring_create(void);
void req_ring_destroy(RequestRing *r);
DoneRing *done_ring_create(void);
void done_ring_destroy(DoneRing *r);
#ifdef __cplusplus
}
#endif
