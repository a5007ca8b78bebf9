/* attention_config.c - shape of the fixed128 decode step (reference
 * cu/attention_decode.cu:48-58). */
#include "attention_decode.h"

DecodeMicrokernelConfig
attention_decode_config_fixed128(void)
{
    DecodeMicrokernelConfig c;
    c.head_dim = DECODE_FIXED_HEAD_DIM;
    c.tokens_per_block = KV_LAYOUT_TOKENS_PER_BLOCK;
    c.tile_tokens = DECODE_TILE_TOKENS;
    c.prefetch_stages = DECODE_PREFETCH_STAGES;
    c.shared_bytes = DECODE_PREFETCH_STAGES * KV_LAYOUT_BLOCK_BYTES;
    return c;
}
