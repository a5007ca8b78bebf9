/*
 * decode_batch.h - host-side grouping of up to 32 descriptors into one ring
 * commit.  Drop-in for reference include/decode_batch.h:7-22.
 * decode_batch_contract() is also usable from device code here (the
 * reference calls a host-only function from its worker, cu/worker.cu:32).
 */
#pragma once
#include <stdint.h>
#include "descriptor.h"
#include "ring.h"

#define DECODE_DESCRIPTOR_BATCH_LIMIT 32U

typedef struct {
    uint32_t count;
    Descriptor descs[DECODE_DESCRIPTOR_BATCH_LIMIT];
} DecodeDispatchBatch;

typedef struct {
    uint16_t batch_size;
    uint16_t batch_index;
} DecodeBatchContract;

#ifdef __cplusplus
extern "C" {
#endif
void decode_batch_reset(DecodeDispatchBatch *batch);
int decode_batch_push(DecodeDispatchBatch *batch, const Descriptor *desc);
int decode_batch_submit(CommandRing *ring, const DecodeDispatchBatch *batch);
DecodeBatchContract decode_batch_contract(const Descriptor *desc);
#ifdef __cplusplus
}
#endif

/* Same contract as decode_batch_contract(), inline for device code. */
static inline RT_HD DecodeBatchContract
decode_batch_contract_inline(const Descriptor *desc)
{
    DecodeBatchContract c;
    c.batch_size = desc ? desc->batch_size : (uint16_t)0;
    c.batch_index = desc ? desc->batch_index : (uint16_t)0;
    return c;
}
