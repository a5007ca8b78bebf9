/* hw_wire.c - the 64-byte completion wire record (hw_desc.h). */
#include <string.h>

#include "hw_desc.h"

void
hw_completion_wire_encode(const hw_desc_t *done, hw_completion_wire_t *wire)
{
    memcpy(wire, done, sizeof(*wire));
    wire->flags = (uint16_t)((done->flags & 0xFFu) |
                             ((uint32_t)hw_completion_status(done) << HW_WIRE_STATUS_SHIFT));
}

void
hw_completion_wire_decode(const hw_completion_wire_t *wire, completion_t *out)
{
    out->rollout_id = (uint16_t)wire->rollout_id;
    out->status = (uint8_t)(wire->flags >> HW_WIRE_STATUS_SHIFT);
    out->final_seq_len = (uint16_t)wire->seq_len;
    out->reward_id = (uint16_t)wire->reward_model_id;
}
