/* reward.c - reward descriptor ring and mock scorer (reference
 * src/reward.c:5-41): producer index prod.head, consumer index cons.tail,
 * 0 / -1 returns, mock score (n & 0xFF) / 255. */
#include "reward.h"

#include <string.h>

void
reward_ring_init(RewardRing *r)
{
    memset(r, 0, sizeof(*r));
}

int
reward_push(RewardRing *r, const RewardDesc *d)
{
    uint32_t h = rt_load_acquire_u32(&r->prod.head);
    uint32_t t = __atomic_load_n(&r->cons.tail, __ATOMIC_RELAXED);
    if ((uint32_t)REWARD_RING_SIZE - (h - t) < 1u)
        return -1;
    r->slots[h & (REWARD_RING_SIZE - 1)] = *d;
    rt_store_release_u32(&r->prod.head, h + 1u);
    return 0;
}

int
reward_pop(RewardRing *r, RewardDesc *d)
{
    uint32_t t = __atomic_load_n(&r->cons.tail, __ATOMIC_ACQUIRE);
    uint32_t h = rt_load_relaxed_u32(&r->prod.head);
    if (t == h)
        return -1;
    *d = r->slots[t & (REWARD_RING_SIZE - 1)];
    __atomic_store_n(&r->cons.tail, t + 1u, __ATOMIC_RELEASE);
    return 0;
}

float
reward_score_mock(const void *tokens, uint32_t n)
{
    (void)tokens;
    return reward_score_mock_inline(n);
}
