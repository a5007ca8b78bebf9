/*
 * attention_decode.h - fixed-shape decode step of the per-step CommandRing
 * path.  Drop-in for reference include/attention_decode.h:23-67 (constants,
 * DecodeStepArgs/Result, DecodeMicrokernelConfig and the config query).
 *
 * The reference's __device__ attention_decode_step_fixed128() is not an
 * exported symbol; its B200 replacement runs inside the persistent decode
 * worker (rlrt.h rt_launch_decode_worker) and as the standalone launcher
 * rt_attention_fixed128().
 */
#pragma once
#include <stdint.h>
#include "descriptor.h"
#include "kv_layout.h"
#include "sample.h"

#define DECODE_FIXED_HEAD_DIM      KV_LAYOUT_HEAD_DIM
#define DECODE_TILE_TOKENS         16U
#define DECODE_PREFETCH_STAGES     3U
#define DECODE_WARPS_PER_BLOCK     1U

typedef enum {
    DECODE_PATH_STUB = 0,
    DECODE_PATH_FIXED128 = 1
} DecodePathKind;

typedef struct {
    const void *q_ptr;     /* fp16[128], or NULL for the synthesized query */
    void       *o_ptr;     /* fp32[128], or NULL */
    uint32_t    seq_len;
    uint32_t    head_dim;
    uint32_t    kv_block_base_idx;
    uint32_t    kv_block_count;
    uint32_t    output_token_offset;
} DecodeStepArgs;

typedef struct {
    uint32_t path_kind;
    uint32_t token_id;
    uint32_t bytes_touched;
    uint32_t tile_count;
    uint64_t cycle_estimate;
} DecodeStepResult;

typedef struct {
    uint32_t head_dim;
    uint32_t tokens_per_block;
    uint32_t tile_tokens;
    uint32_t prefetch_stages;
    uint32_t shared_bytes;
} DecodeMicrokernelConfig;

RT_STATIC_ASSERT(sizeof(DecodeStepResult) == 24, "DecodeStepResult layout");
RT_STATIC_ASSERT(sizeof(DecodeMicrokernelConfig) == 20, "DecodeMicrokernelConfig layout");

#ifdef __cplusplus
extern "C" {
#endif
DecodeMicrokernelConfig attention_decode_config_fixed128(void);
#ifdef __cplusplus
}
#endif
