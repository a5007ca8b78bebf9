/* arena.c - KV arena in HBM.
 *
 * Same API and allocation order as reference src/arena.c:7-58 (lowest free
 * block first, -1 when exhausted, release(-1) ignored, abort when the
 * memory cannot be obtained).  The blocks live in device memory, zeroed at
 * init so every KV page holds finite values before first use.  Unlike the
 * reference, acquire never hands out a block index past
 * capacity / block_size: such a block would address memory outside the
 * allocation. */
#include "arena.h"

#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <cuda_runtime_api.h>

static uint64_t
arena_block_limit(const KVArena *a)
{
    uint64_t n = a->block_size ? (uint64_t)(a->capacity / a->block_size) : 0u;
    uint64_t cap = (uint64_t)BITMAP_WORDS * 64u;
    return n < cap ? n : cap;
}

void
arena_init(KVArena *a, size_t capacity, size_t block_size)
{
    void *p = NULL;
    cudaError_t err;

    a->capacity = capacity;
    a->block_size = block_size;
    a->base = NULL;
    memset(a->bitmap, 0, sizeof(a->bitmap));

    err = cudaMalloc(&p, capacity);
    if (err != cudaSuccess) {
        fprintf(stderr, "arena_init: cudaMalloc(%zu) failed: %s\n",
                capacity, cudaGetErrorString(err));
        abort();
    }
    err = cudaMemset(p, 0, capacity);
    if (err == cudaSuccess)
        err = cudaDeviceSynchronize();
    if (err != cudaSuccess) {
        fprintf(stderr, "arena_init: zero-fill failed: %s\n", cudaGetErrorString(err));
        abort();
    }
    a->base = (uint8_t *)p;
}

int64_t
arena_acquire(KVArena *a)
{
    uint64_t limit = arena_block_limit(a);
    uint64_t words = (limit + 63u) / 64u;
    for (uint64_t w = 0; w < words; w++) {
        uint64_t free_bits = ~a->bitmap[w];
        if (free_bits) {
            uint64_t idx = w * 64u + (uint64_t)__builtin_ctzll(free_bits);
            if (idx >= limit)
                return -1;
            a->bitmap[w] |= 1ull << (idx & 63u);
            return (int64_t)idx;
        }
    }
    return -1;
}

void
arena_release(KVArena *a, int64_t idx)
{
    if (idx < 0 || (uint64_t)idx >= (uint64_t)BITMAP_WORDS * 64u)
        return;
    a->bitmap[idx / 64] &= ~(1ull << (idx % 64));
}

void
arena_destroy(KVArena *a)
{
    if (a->base)
        cudaFree(a->base);
    a->base = NULL;
}
