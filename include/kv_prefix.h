/*
 * kv_prefix.h - copy-on-write prefix sharing table.
 *
 * Drop-in for reference include/kv_prefix.h:6-56 and src/kv_prefix.c:5-149:
 * 512 refcounted prefixes, 16,384 branches (2 x MAX_ROLLOUTS), free bitmaps
 * with 1 = free, lowest-id-first allocation, 0 / -1 returns.
 *
 * The packed records are 28 and 36 bytes.  The reference asserts 24 and 28
 * (reference include/kv_prefix.h:18,31), which is false for the fields it
 * declares, so its table does not compile as shipped; the field layout is
 * kept and the true sizes are asserted here.
 */
#pragma once
#include <stddef.h>
#include <stdint.h>
#include "rt_sync.h"

#define MAX_ROLLOUTS 8192
#define MAX_PREFIXES 512
#define MAX_BRANCHES (MAX_ROLLOUTS * 2)

typedef struct __attribute__((packed)) {
    uint32_t prefix_id;
    uint32_t refcnt;
    int64_t  kv_block_offset;   /* -1 once released */
    uint32_t token_len;
    uint32_t kv_block_count;
    uint32_t flags;
} KVPrefix;

typedef struct __attribute__((packed)) {
    uint32_t branch_id;
    uint32_t rollout_id;
    uint32_t prefix_id;
    int64_t  delta_kv_offset;
    uint32_t delta_len;
    uint32_t delta_block_count;
    uint32_t state;
    uint32_t flags;
} KVBranch;

RT_STATIC_ASSERT(sizeof(KVPrefix) == 28, "KVPrefix packed size");
RT_STATIC_ASSERT(sizeof(KVBranch) == 36, "KVBranch packed size");

typedef struct {
    KVPrefix prefixes[MAX_PREFIXES];
    uint64_t prefix_bitmap[(MAX_PREFIXES + 63) / 64];   /* 1 = free */
    KVBranch branches[MAX_BRANCHES];
    uint64_t branch_bitmap[(MAX_BRANCHES + 63) / 64];   /* 1 = free */
    uint32_t next_branch_id;
} KVPrefixTable;

#ifdef __cplusplus
extern "C" {
#endif
void  kv_prefix_table_init(KVPrefixTable *t);
int   kv_prefix_register(KVPrefixTable *t, int64_t kv_offset,
                         uint32_t token_len, uint32_t nblocks,
                         uint32_t *out_id);
int   kv_prefix_acquire(KVPrefixTable *t, uint32_t prefix_id);
int   kv_prefix_release(KVPrefixTable *t, uint32_t prefix_id);
KVPrefix *kv_prefix_get(KVPrefixTable *t, uint32_t prefix_id);

int   kv_branch_alloc(KVPrefixTable *t, uint32_t rollout_id,
                      uint32_t prefix_id, int64_t delta_kv_offset,
                      uint32_t delta_len, uint32_t delta_blocks,
                      uint32_t *out_branch_id);
int   kv_branch_free(KVPrefixTable *t, uint32_t branch_id);
KVBranch *kv_branch_get(KVPrefixTable *t, uint32_t branch_id);

int64_t kv_branch_total_offset(KVPrefixTable *t, uint32_t branch_id);
#ifdef __cplusplus
}
#endif
