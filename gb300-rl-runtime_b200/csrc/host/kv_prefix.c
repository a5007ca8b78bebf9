/* kv_prefix.c - host side of copy-on-write prefix sharing.
 *
 * Contract of reference src/kv_prefix.c:5-149: lowest free id first, a new
 * prefix starts with refcnt 1, the last release poisons kv_block_offset to
 * -1 and returns the id to the free set, a branch holds one reference on its
 * prefix, and kv_branch_total_offset() returns the prefix's offset (the
 * branch's own delta only when the prefix id is out of range).  The device
 * side (page-table resolution for the rollout worker) is rt_kv_branch_resolve
 * in rlrt.h. */
#include "kv_prefix.h"

#include <string.h>

static void
bitmap_set_all_free(uint64_t *bm, uint32_t words, uint32_t n_ids)
{
    for (uint32_t w = 0; w < words; w++)
        bm[w] = ~0ull;
    if (n_ids % 64u)
        bm[n_ids / 64u] &= (1ull << (n_ids % 64u)) - 1u;
}

static int
bitmap_take_lowest(uint64_t *bm, uint32_t words, uint32_t *out_id)
{
    for (uint32_t w = 0; w < words; w++) {
        if (bm[w]) {
            uint32_t b = (uint32_t)__builtin_ctzll(bm[w]);
            bm[w] &= ~(1ull << b);
            *out_id = w * 64u + b;
            return 0;
        }
    }
    return -1;
}

static void
bitmap_give_back(uint64_t *bm, uint32_t id)
{
    bm[id / 64u] |= 1ull << (id % 64u);
}

#define PREFIX_WORDS ((uint32_t)(sizeof(((KVPrefixTable *)0)->prefix_bitmap) / sizeof(uint64_t)))
#define BRANCH_WORDS ((uint32_t)(sizeof(((KVPrefixTable *)0)->branch_bitmap) / sizeof(uint64_t)))

void
kv_prefix_table_init(KVPrefixTable *t)
{
    memset(t, 0, sizeof(*t));
    bitmap_set_all_free(t->prefix_bitmap, PREFIX_WORDS, MAX_PREFIXES);
    bitmap_set_all_free(t->branch_bitmap, BRANCH_WORDS, MAX_BRANCHES);
}

int
kv_prefix_register(KVPrefixTable *t, int64_t kv_offset, uint32_t token_len,
                   uint32_t nblocks, uint32_t *out_id)
{
    uint32_t id;
    KVPrefix *p;

    if (bitmap_take_lowest(t->prefix_bitmap, PREFIX_WORDS, &id) != 0)
        return -1;
    p = &t->prefixes[id];
    p->prefix_id = id;
    p->refcnt = 1u;
    p->kv_block_offset = kv_offset;
    p->token_len = token_len;
    p->kv_block_count = nblocks;
    p->flags = 0u;
    *out_id = id;
    return 0;
}

int
kv_prefix_acquire(KVPrefixTable *t, uint32_t prefix_id)
{
    KVPrefix *p;
    if (prefix_id >= MAX_PREFIXES)
        return -1;
    p = &t->prefixes[prefix_id];
    if (p->refcnt == 0u)
        return -1;
    p->refcnt++;
    return 0;
}

int
kv_prefix_release(KVPrefixTable *t, uint32_t prefix_id)
{
    KVPrefix *p;
    if (prefix_id >= MAX_PREFIXES)
        return -1;
    p = &t->prefixes[prefix_id];
    if (p->refcnt == 0u)
        return -1;
    if (--p->refcnt == 0u) {
        p->kv_block_offset = -1;
        p->token_len = 0u;
        bitmap_give_back(t->prefix_bitmap, prefix_id);
    }
    return 0;
}

KVPrefix *
kv_prefix_get(KVPrefixTable *t, uint32_t prefix_id)
{
    return prefix_id < MAX_PREFIXES ? &t->prefixes[prefix_id] : NULL;
}

int
kv_branch_alloc(KVPrefixTable *t, uint32_t rollout_id, uint32_t prefix_id,
                int64_t delta_kv_offset, uint32_t delta_len,
                uint32_t delta_blocks, uint32_t *out_branch_id)
{
    uint32_t id;
    KVBranch *b;

    if (bitmap_take_lowest(t->branch_bitmap, BRANCH_WORDS, &id) != 0)
        return -1;
    b = &t->branches[id];
    b->branch_id = id;
    b->rollout_id = rollout_id;
    b->prefix_id = prefix_id;
    b->delta_kv_offset = delta_kv_offset;
    b->delta_len = delta_len;
    b->delta_block_count = delta_blocks;
    b->state = 0u;
    b->flags = 0u;
    (void)kv_prefix_acquire(t, prefix_id);  /* result not propagated, as in the reference */
    *out_branch_id = id;
    return 0;
}

int
kv_branch_free(KVPrefixTable *t, uint32_t branch_id)
{
    KVBranch *b;
    if (branch_id >= MAX_BRANCHES)
        return -1;
    b = &t->branches[branch_id];
    (void)kv_prefix_release(t, b->prefix_id);
    b->rollout_id = UINT32_MAX;
    bitmap_give_back(t->branch_bitmap, branch_id);
    return 0;
}

KVBranch *
kv_branch_get(KVPrefixTable *t, uint32_t branch_id)
{
    return branch_id < MAX_BRANCHES ? &t->branches[branch_id] : NULL;
}

int64_t
kv_branch_total_offset(KVPrefixTable *t, uint32_t branch_id)
{
    KVBranch *b;
    KVPrefix *p;
    if (branch_id >= MAX_BRANCHES)
        return -1;
    b = &t->branches[branch_id];
    p = kv_prefix_get(t, b->prefix_id);
    return p ? p->kv_block_offset : b->delta_kv_offset;
}
