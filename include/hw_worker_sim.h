/*
 * hw_worker_sim.h - CPU model of the descriptor engine (consumer of cmdq,
 * producer of doneq).  Drop-in for reference include/hw_worker_sim.h:6-14.
 */
#pragma once
#include <stdint.h>
#include "hw_ring.h"

typedef struct {
    hw_ring_t *cmdq;
    hw_ring_t *doneq;
    volatile uint32_t *stop;
    uint64_t decoded_tokens;
    uint64_t completions;
} hw_worker_sim_t;

#ifdef __cplusplus
extern "C" {
#endif
void hw_worker_sim_run(hw_worker_sim_t *worker);
#ifdef __cplusplus
}
#endif
