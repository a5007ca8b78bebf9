/* hw_worker_sim.c - CPU model of the descriptor engine.
 *
 * Semantics of reference src/hw_worker_sim.c:22-59 for every descriptor:
 *   STOP                 -> leave the loop, no completion
 *   opcode != DECODE     -> dropped, no completion
 *   seq_len >= max       -> echoed unchanged (no flags, no tokens)
 *   otherwise advance seq_len one token at a time until it reaches
 *   max_tokens (DONE) or the next multiple of 32 (NEEDS_REWARD); DONE wins
 *   when both coincide.  The whole updated descriptor goes to doneq, with a
 *   spin while doneq is full.
 * The token run is computed in closed form rather than one token per
 * iteration; the resulting descriptor stream is identical. */
#include "hw_worker_sim.h"

static inline void
hw_cpu_relax(void)
{
#if defined(__x86_64__)
    __asm__ volatile("pause" ::: "memory");
#elif defined(__aarch64__)
    __asm__ volatile("yield" ::: "memory");
#endif
}

/* Advance one DECODE descriptor to its next stopping point; returns the
 * number of tokens decoded. */
static uint32_t
hw_decode_advance(hw_desc_t *d)
{
    uint64_t pos = d->seq_len;
    uint64_t boundary;

    if (pos >= d->max_tokens)
        return 0u;
    boundary = (pos | (uint64_t)(HW_REWARD_BOUNDARY - 1u)) + 1u;
    if ((uint64_t)d->max_tokens <= boundary) {
        d->seq_len = d->max_tokens;
        d->flags |= (uint16_t)DESC_FLAG_DONE;
    } else {
        d->seq_len = (uint32_t)boundary;
        d->flags |= (uint16_t)DESC_FLAG_NEEDS_REWARD;
    }
    return (uint32_t)(d->seq_len - pos);
}

void
hw_worker_sim_run(hw_worker_sim_t *worker)
{
    while (!rt_load_acquire_u32(worker->stop)) {
        hw_desc_t d;

        if (hw_ring_pop(worker->cmdq, &d) != 0) {
            hw_cpu_relax();
            continue;
        }
        if (d.opcode == DESC_OP_STOP)
            break;
        if (d.opcode != DESC_OP_DECODE)
            continue;

        worker->decoded_tokens += hw_decode_advance(&d);

        while (hw_ring_push(worker->doneq, &d) != 0)
            hw_cpu_relax();
        worker->completions++;
    }
}
