/* decode_batch.c - up to 32 descriptors published with one ring commit,
 * each stamped with (batch_size, batch_index).  Contract of reference
 * src/decode_batch.c:3-51: push/submit return 0 / -1, submit fails without
 * writing anything when the ring lacks room for the whole window. */
#include "decode_batch.h"

void
decode_batch_reset(DecodeDispatchBatch *batch)
{
    if (batch)
        batch->count = 0;
}

int
decode_batch_push(DecodeDispatchBatch *batch, const Descriptor *desc)
{
    if (batch == NULL || desc == NULL || batch->count >= DECODE_DESCRIPTOR_BATCH_LIMIT)
        return -1;
    batch->descs[batch->count] = *desc;
    batch->count++;
    return 0;
}

int
decode_batch_submit(CommandRing *ring, const DecodeDispatchBatch *batch)
{
    uint32_t pos, n, i;

    if (ring == NULL || batch == NULL || batch->count == 0)
        return -1;
    n = batch->count;
    pos = ring_acquire(ring, n);
    if (pos == UINT32_MAX)
        return -1;
    for (i = 0; i < n; i++) {
        Descriptor *slot = &ring->slots[(pos + i) & (RING_SIZE - 1u)];
        *slot = batch->descs[i];
        slot->batch_size = (uint16_t)n;
        slot->batch_index = (uint16_t)i;
    }
    ring_commit(ring, n);
    return 0;
}

DecodeBatchContract
decode_batch_contract(const Descriptor *desc)
{
    return decode_batch_contract_inline(desc);
}
