/*
 * hw_desc.h - the 64-byte hardware descriptor and its completion view.
 *
 * Drop-in for reference include/hw_desc.h:1-35.  Field order, widths, the
 * packed/64-byte-aligned layout and every opcode/flag value are part of the
 * wire contract with callers and are kept identical; the offsets are pinned
 * by the static asserts at the end of this file.
 */
#pragma once
#include <stddef.h>
#include <stdint.h>
#include "rt_sync.h"

#define DESC_OP_DECODE       1U
#define DESC_OP_REWARD       2U
#define DESC_OP_PREFILL      3U
#define DESC_OP_STOP         255U

#define DESC_FLAG_NEEDS_REWARD (1u << 0)
#define DESC_FLAG_DONE         (1u << 1)
#define DESC_FLAG_COW_PREFIX   (1u << 2)

/* Reward boundary of the worker: a decode run stops every 32 tokens. */
#define HW_REWARD_BOUNDARY     32u

typedef struct __attribute__((packed, aligned(64))) {
    uint16_t opcode;             /* DESC_OP_* */
    uint16_t flags;              /* DESC_FLAG_* */
    uint32_t rollout_id;
    uint32_t kv_arena_id;
    uint32_t prefix_id;          /* 0 = no shared prefix */
    uint64_t kv_offset;
    uint64_t delta_offset;
    uint32_t seq_len;            /* tokens decoded so far */
    uint32_t max_tokens;
    uint32_t reward_model_id;
    uint32_t reserved0;          /* submit path stores the GPU group id */
    uint64_t user_data;
    uint64_t checksum_or_cookie;
} hw_desc_t;

RT_STATIC_ASSERT(sizeof(hw_desc_t) == 64, "hw_desc_t must be one cache line");
RT_STATIC_ASSERT(offsetof(hw_desc_t, rollout_id) == 4, "hw_desc_t layout");
RT_STATIC_ASSERT(offsetof(hw_desc_t, kv_offset) == 16, "hw_desc_t layout");
RT_STATIC_ASSERT(offsetof(hw_desc_t, seq_len) == 32, "hw_desc_t layout");
RT_STATIC_ASSERT(offsetof(hw_desc_t, reward_model_id) == 40, "hw_desc_t layout");
RT_STATIC_ASSERT(offsetof(hw_desc_t, user_data) == 48, "hw_desc_t layout");
RT_STATIC_ASSERT(offsetof(hw_desc_t, checksum_or_cookie) == 56, "hw_desc_t layout");

/*
 * completion_t - compact completion record of the descriptor engine
 * (reference rtl/desc_pkg.sv:22-31: rollout_id 16 b, status 8 b,
 * final_seq_len 16 b, reward_id 16 b).  The C done ring carries whole
 * updated hw_desc_t records (reference src/hw_worker_sim.c:54); this is the
 * byte-packed host view of one of them, filled by hw_completion_from_desc().
 */
#define HW_COMP_STATUS_DONE           0x01u
#define HW_COMP_STATUS_REWARD_NEEDED  0x02u
#define HW_COMP_STATUS_STOPPED        0xFFu

typedef struct __attribute__((packed)) {
    uint16_t rollout_id;
    uint8_t  status;
    uint16_t final_seq_len;
    uint16_t reward_id;
} completion_t;

RT_STATIC_ASSERT(sizeof(completion_t) == 7, "completion_t is 56 bits");

/* Derive the compact completion from a done-ring descriptor.  DONE takes
 * precedence over REWARD_NEEDED, as in the RTL FSM (reference
 * rtl/rollout_worker_fsm.sv:61-75); a STOP descriptor maps to STOPPED.
 * A descriptor with neither flag (echoed unchanged) reports status 0. */
static inline RT_HD uint8_t
hw_completion_status(const hw_desc_t *d)
{
    if (d->opcode == DESC_OP_STOP)
        return (uint8_t)HW_COMP_STATUS_STOPPED;
    if (d->flags & DESC_FLAG_DONE)
        return (uint8_t)HW_COMP_STATUS_DONE;
    if (d->flags & DESC_FLAG_NEEDS_REWARD)
        return (uint8_t)HW_COMP_STATUS_REWARD_NEEDED;
    return 0;
}

static inline RT_HD void
hw_completion_from_desc(const hw_desc_t *d, completion_t *out)
{
    out->rollout_id = (uint16_t)d->rollout_id;
    out->status = hw_completion_status(d);
    out->final_seq_len = (uint16_t)d->seq_len;
    out->reward_id = (uint16_t)d->reward_model_id;
}

/*
 * hw_completion_wire_t - one 64-byte completion record for both the C done
 * ring and a 512-bit RTL completion output (the byte-identical completion
 * definition the reference lists as a gap, docs/descriptor_contract.md
 * "Gaps To Close" 2 and the 64-byte roadmap).  It is the done descriptor
 * itself, every field at its hw_desc_t offset, with the completion status
 * (HW_COMP_STATUS_*, one namespace with the RTL's completion_t) in the high
 * byte of `flags`, which the descriptor flags (bits 0-2) leave free; the
 * compact completion_t is derived from it without loss of its fields.
 */
typedef hw_desc_t hw_completion_wire_t;
#define HW_WIRE_STATUS_SHIFT 8u

#ifdef __cplusplus
extern "C" {
#endif
/* Encode a done descriptor as a wire record; decode a wire record into the
 * compact completion_t (equal to hw_completion_from_desc of the descriptor). */
void hw_completion_wire_encode(const hw_desc_t *done, hw_completion_wire_t *wire);
void hw_completion_wire_decode(const hw_completion_wire_t *wire, completion_t *out);
#ifdef __cplusplus
}
#endif
