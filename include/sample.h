/*
 * sample.h - per-trajectory sampling parameters.
 * Drop-in for reference include/sample.h:11-29 (same SampleState layout and
 * MAX_VOCAB_SIZE).  The reference's device functions sample_init() and
 * sample_token() are replaced by the fused row sampler rt_sample_rows()
 * declared in rlrt.h, which draws its uniform from a counter-based Philox
 * stream instead of the xoshiro256** state kept here.
 */
#pragma once
#include <stddef.h>
#include <stdint.h>
#include "rt_sync.h"

#define MAX_VOCAB_SIZE 131072

typedef struct {
    uint64_t rng_state[4];
    float    temperature;
    uint16_t top_k;
    float    top_p;
    uint32_t vocab_size;
} SampleState;

RT_STATIC_ASSERT(sizeof(SampleState) == 48, "SampleState natural layout");
RT_STATIC_ASSERT(offsetof(SampleState, top_p) == 40, "SampleState layout");
