/*
 * kv_layout.h - KV memory layouts.
 *
 * Part 1 keeps the reference's fixed-shape block (reference
 * include/kv_layout.h:15-80): one head of d=128, 32 tokens, K plane then V
 * plane, 2-byte scalars, 16 KiB per block.  It is used by the per-step
 * CommandRing decode path.
 *
 * Part 2 is the paged GQA layout of the rollout path (new; the reference
 * has no paging).  One page holds RT_PAGE_TOKENS consecutive tokens of one
 * sequence for every KV head:
 *
 *     page p, kv head h, plane (0 = K, 1 = V), token t, dim d  ->
 *     bf16 element  ((((p * Hkv + h) * 2 + plane) * 16 + t) * D + d)
 *
 * so each (page, head, plane) is a contiguous 16 x 128 bf16 tile of 4 KiB
 * whose rows are 256 B: exactly the box a TMA tensor copy moves in two
 * 128-byte-swizzled halves.  A page of the benchmark shape (Hkv = 8, D = 128)
 * is 64 KiB.  Page tables are int32 page indices, one row per sequence.
 */
#pragma once
#include <stddef.h>
#include <stdint.h>
#include "rt_sync.h"

#define KV_LAYOUT_HEAD_DIM         128U
#define KV_LAYOUT_TOKENS_PER_BLOCK 32U
#define KV_LAYOUT_SCALAR_BYTES     2U
#define KV_LAYOUT_VEC_BYTES        16U
#define KV_LAYOUT_ALIGNMENT        128U

#define KV_LAYOUT_K_BYTES \
    (KV_LAYOUT_TOKENS_PER_BLOCK * KV_LAYOUT_HEAD_DIM * KV_LAYOUT_SCALAR_BYTES)
#define KV_LAYOUT_V_BYTES KV_LAYOUT_K_BYTES
#define KV_LAYOUT_BLOCK_BYTES (KV_LAYOUT_K_BYTES + KV_LAYOUT_V_BYTES)

typedef struct {
    uint32_t token_count;
    uint32_t head_dim;
    uint32_t scalar_bytes;
    uint32_t vec_bytes;
    uint32_t k_stride_bytes;
    uint32_t v_stride_bytes;
    uint32_t block_bytes;
    uint32_t alignment;
} KvLayoutDesc;

RT_STATIC_ASSERT((KV_LAYOUT_HEAD_DIM * KV_LAYOUT_SCALAR_BYTES) % KV_LAYOUT_VEC_BYTES == 0,
                 "head rows must split into 16-byte vectors");
RT_STATIC_ASSERT(KV_LAYOUT_BLOCK_BYTES % KV_LAYOUT_ALIGNMENT == 0,
                 "blocks keep 128-byte alignment");

static inline RT_HD KvLayoutDesc
kv_layout_desc_fixed128(void)
{
    KvLayoutDesc d;
    d.token_count = KV_LAYOUT_TOKENS_PER_BLOCK;
    d.head_dim = KV_LAYOUT_HEAD_DIM;
    d.scalar_bytes = KV_LAYOUT_SCALAR_BYTES;
    d.vec_bytes = KV_LAYOUT_VEC_BYTES;
    d.k_stride_bytes = KV_LAYOUT_HEAD_DIM * KV_LAYOUT_SCALAR_BYTES;
    d.v_stride_bytes = KV_LAYOUT_HEAD_DIM * KV_LAYOUT_SCALAR_BYTES;
    d.block_bytes = KV_LAYOUT_BLOCK_BYTES;
    d.alignment = KV_LAYOUT_ALIGNMENT;
    return d;
}

static inline RT_HD uint32_t
kv_layout_block_offset_bytes(uint32_t block_idx)
{
    return block_idx * KV_LAYOUT_BLOCK_BYTES;
}

static inline RT_HD uint32_t
kv_layout_k_offset_bytes(uint32_t token_idx)
{
    return token_idx * (KV_LAYOUT_HEAD_DIM * KV_LAYOUT_SCALAR_BYTES);
}

static inline RT_HD uint32_t
kv_layout_v_plane_base_bytes(void)
{
    return KV_LAYOUT_K_BYTES;
}

static inline RT_HD uint32_t
kv_layout_v_offset_bytes(uint32_t token_idx)
{
    return kv_layout_v_plane_base_bytes() + kv_layout_k_offset_bytes(token_idx);
}

/* ---- paged GQA layout (rollout path) ---------------------------------- */
#define RT_PAGE_TOKENS   16u
#define RT_HEAD_DIM      128u

/* bf16 elements from the arena base to (page, head, plane, token, 0). */
static inline RT_HD uint64_t
rt_page_elem_offset(uint64_t page, uint32_t head, uint32_t plane,
                    uint32_t token, uint32_t num_kv_heads)
{
    return ((((page * num_kv_heads + head) * 2u + plane) * RT_PAGE_TOKENS + token)
            * (uint64_t)RT_HEAD_DIM);
}

/* Bytes of one page for all KV heads. */
static inline RT_HD uint64_t
rt_page_bytes(uint32_t num_kv_heads)
{
    return (uint64_t)num_kv_heads * 2u * RT_PAGE_TOKENS * RT_HEAD_DIM * 2u;
}
