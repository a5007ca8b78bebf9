/*
 * descriptor.h - 32-byte per-step decode descriptor of the CommandRing.
 * Drop-in for reference include/descriptor.h:5-23 (same constants, field
 * order and packed layout).
 */
#pragma once
#include <stddef.h>
#include <stdint.h>
#include "rt_sync.h"

#define RING_SIZE              4096
#define MAX_KV_BLOCKS_PER_STEP 64
#define DESCRIPTOR_ALIGN       128

#pragma pack(push, 1)
typedef struct {
    uint64_t seq_id;              /* trajectory id; UINT64_MAX = worker stop */
    uint32_t kv_block_offset;     /* arena block index */
    uint16_t num_kv_blocks;
    uint8_t  attention_flags;
    uint8_t  pad;
    uint32_t output_token_offset; /* q/o io slot */
    uint64_t reward_cookie;
    uint16_t batch_size;          /* stamped by decode_batch_submit */
    uint16_t batch_index;
} Descriptor;
#pragma pack(pop)

RT_STATIC_ASSERT(sizeof(Descriptor) == 32, "Descriptor must be 32 bytes");
RT_STATIC_ASSERT(offsetof(Descriptor, output_token_offset) == 16, "Descriptor layout");
RT_STATIC_ASSERT(offsetof(Descriptor, batch_size) == 28, "Descriptor layout");
