/* infer_submit.c - build one DECODE descriptor, publish it, ring the
 * doorbell with the new tail.  Field-for-field the contract of reference
 * src/infer_submit.c:3-37: COW flag iff a prefix id is given, reserved0 =
 * GPU group, user_data = rollout id, cookie = kv ^ delta ^ (rollout << 32). */
#include "infer_submit.h"

#include <string.h>

int
infer_submit_decode(infer_hw_ctx_t *ctx,
                    uint32_t rollout_id,
                    uint64_t kv_offset,
                    uint64_t delta_offset,
                    uint32_t prefix_id,
                    uint32_t seq_len,
                    uint32_t max_tokens)
{
    hw_desc_t d;

    if (ctx == NULL || ctx->cmdq == NULL || ctx->doorbell == NULL)
        return -1;

    memset(&d, 0, sizeof(d));
    d.opcode = (uint16_t)DESC_OP_DECODE;
    d.flags = (uint16_t)(prefix_id != 0u ? DESC_FLAG_COW_PREFIX : 0u);
    d.rollout_id = rollout_id;
    d.kv_arena_id = ctx->kv_arena_id;
    d.prefix_id = prefix_id;
    d.kv_offset = kv_offset;
    d.delta_offset = delta_offset;
    d.seq_len = seq_len;
    d.max_tokens = max_tokens;
    d.reward_model_id = 0u;
    d.reserved0 = ctx->gpu_group_id;
    d.user_data = (uint64_t)rollout_id;
    d.checksum_or_cookie = kv_offset ^ delta_offset ^ ((uint64_t)rollout_id << 32);

    if (hw_ring_push(ctx->cmdq, &d) != 0)
        return -1;

    mmio_write32(ctx->doorbell, rt_load_acquire_u32(&ctx->cmdq->tail));
    return 0;
}
