/*
 * arena.h - KV block arena.  Drop-in for reference include/arena.h:5-35 and
 * src/arena.c:7-58: same struct (base, capacity, block_size, 1 Mi-block
 * bitmap with 1 = in use), lowest-free-block-first acquire returning the
 * index or -1, release of a negative index is a no-op, init aborts when the
 * memory cannot be obtained.
 *
 * B200 difference: `base` is device memory (HBM, cudaMalloc), zero-filled at
 * init, so KV pages are read by kernels at HBM bandwidth instead of across
 * the host link.  arena_block_ptr() therefore yields a device address; the
 * bitmap stays in host memory and is managed by host code only.
 */
#pragma once
#include <stddef.h>
#include <stdint.h>
#include "rt_sync.h"

#define BITMAP_WORDS ((1UL << 20) / 64)  /* up to 1 Mi blocks */

typedef struct {
    uint8_t *base;        /* device address of block 0 */
    size_t   capacity;    /* bytes */
    size_t   block_size;  /* bytes per block */
    uint64_t bitmap[BITMAP_WORDS];
} KVArena;

#ifdef __cplusplus
extern "C" {
#endif
void    arena_init(KVArena *a, size_t capacity, size_t block_size);
int64_t arena_acquire(KVArena *a);
void    arena_release(KVArena *a, int64_t idx);
void    arena_destroy(KVArena *a);
#ifdef __cplusplus
}
#endif

static inline RT_HD uint8_t *
arena_block_ptr(KVArena *a, int64_t idx)
{
    return a->base + idx * (int64_t)a->block_size;
}
