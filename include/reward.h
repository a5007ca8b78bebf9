/*
 * reward.h - reward descriptor ring and the mock scorer.
 * Drop-in for reference include/reward.h:4-32 and src/reward.c:5-41: the
 * 24-byte RewardDesc, 1,024-slot ring whose producer index is prod.head and
 * consumer index cons.tail, push/pop -> 0/-1, reward_score_mock(n) =
 * (n & 0xFF) / 255.
 *
 * Group-normalised advantages and the cross-GPU reward allgather are new in
 * this runtime and are declared in rlrt.h (rt_grpo_advantages,
 * rt_reward_allgather).
 */
#pragma once
#include <stddef.h>
#include <stdint.h>
#include "rt_sync.h"

#define REWARD_RING_SIZE 1024

typedef struct __attribute__((packed)) {
    uint32_t rollout_id;
    uint32_t token_start;
    uint32_t token_count;
    uint32_t reward_model_id;
    float    reward;
    uint32_t flags;
} RewardDesc;

RT_STATIC_ASSERT(sizeof(RewardDesc) == 24, "RewardDesc must be 24 bytes");

typedef struct __attribute__((packed)) {
    __attribute__((aligned(64))) volatile uint32_t head;
    uint32_t tail;
    uint8_t  pad[56];
} RewardIndex;

typedef struct {
    __attribute__((aligned(64))) RewardIndex prod;
    __attribute__((aligned(64))) RewardIndex cons;
    __attribute__((aligned(128))) RewardDesc slots[REWARD_RING_SIZE];
} RewardRing;

RT_STATIC_ASSERT(sizeof(RewardIndex) == 64, "RewardIndex is one cache line");
RT_STATIC_ASSERT(offsetof(RewardRing, slots) == 128, "RewardRing layout");

#ifdef __cplusplus
extern "C" {
#endif
void  reward_ring_init(RewardRing *r);
int   reward_push(RewardRing *r, const RewardDesc *d);
int   reward_pop(RewardRing *r, RewardDesc *d);
float reward_score_mock(const void *tokens, uint32_t n);
#ifdef __cplusplus
}
#endif

/* Mock score used on the device by the rollout worker's done path
 * (reference cu/gpu_scheduler.cu:68 and cu/reward.cu:11). */
static inline RT_HD float
reward_score_mock_inline(uint32_t n)
{
    return (float)(n & 0xFFu) / 255.0f;
}
