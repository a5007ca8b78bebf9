/* pump.c - host producer/consumer for a ring-fed GPU rollout run. */
#define _POSIX_C_SOURCE 200112L
#include <string.h>
#include <time.h>

#include "rlrt.h"

static uint64_t
pump_now_ms(void)
{
    struct timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return (uint64_t)ts.tv_sec * 1000u + (uint64_t)ts.tv_nsec / 1000000u;
}

int64_t
rt_host_pump(RequestRing *rq, const RolloutRequest *reqs, uint32_t n, DoneRing *dn,
             RolloutDone *dones, uint32_t n_expected, int send_sentinel, uint32_t timeout_ms)
{
    uint32_t pushed = 0, drained = 0;
    int sentinel_sent = !send_sentinel;
    const uint64_t t0 = pump_now_ms();

    if (!rq || !dn || (n && !reqs) || (n_expected && !dones))
        return -1;
    while (drained < n_expected || pushed < n || !sentinel_sent) {
        int progress = 0;
        while (pushed < n) {
            uint32_t pos = req_ring_acquire(rq);
            if (pos == UINT32_MAX)
                break;
            rq->slots[pos] = reqs[pushed++];
            req_ring_commit(rq);
            progress = 1;
        }
        if (pushed == n && !sentinel_sent && drained >= n_expected) {
            uint32_t pos = req_ring_acquire(rq);
            if (pos != UINT32_MAX) {
                RolloutRequest s;
                memset(&s, 0, sizeof(s));
                s.request_id = RT_REQUEST_SENTINEL;
                rq->slots[pos] = s;
                req_ring_commit(rq);
                sentinel_sent = 1;
                progress = 1;
            }
        }
        while (drained < n_expected && done_ring_pop(dn, &dones[drained]))
            drained++, progress = 1;
        if (!progress) {
            if (timeout_ms && pump_now_ms() - t0 > timeout_ms)
                return -1;
#if defined(__x86_64__)
            __asm__ volatile("pause" ::: "memory");
#endif
        }
    }
    return (int64_t)drained;
}

static uint64_t
pump_now_ns(void)
{
    struct timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return (uint64_t)ts.tv_sec * 1000000000ull + (uint64_t)ts.tv_nsec;
}

/* Open-loop producer: request i enters the ring once the clock has passed
 * its arrival (and the ring has room), so the device sees the arrival
 * process itself, not the ring's backlog.  The consumer side is
 * rt_host_pump's, with a time stamp per drained record. */
int64_t
rt_host_pump_paced(RequestRing *rq, const RolloutRequest *reqs, const uint64_t *arrival_ns,
                   uint32_t n, DoneRing *dn, RolloutDone *dones, uint64_t *done_ns,
                   uint32_t n_expected, int send_sentinel, uint32_t timeout_ms)
{
    uint32_t pushed = 0, drained = 0;
    int sentinel_sent = !send_sentinel;
    const uint64_t t0 = pump_now_ns();
    uint64_t last_progress = t0;

    if (!rq || !dn || (n && !reqs) || (n_expected && !dones))
        return -1;
    while (drained < n_expected || pushed < n || !sentinel_sent) {
        int progress = 0;
        uint64_t now = pump_now_ns();
        while (pushed < n && (!arrival_ns || now - t0 >= arrival_ns[pushed])) {
            uint32_t pos = req_ring_acquire(rq);
            if (pos == UINT32_MAX)
                break;
            rq->slots[pos] = reqs[pushed++];
            req_ring_commit(rq);
            progress = 1;
        }
        if (pushed == n && !sentinel_sent && drained >= n_expected) {
            uint32_t pos = req_ring_acquire(rq);
            if (pos != UINT32_MAX) {
                RolloutRequest s;
                memset(&s, 0, sizeof(s));
                s.request_id = RT_REQUEST_SENTINEL;
                rq->slots[pos] = s;
                req_ring_commit(rq);
                sentinel_sent = 1;
                progress = 1;
            }
        }
        while (drained < n_expected && done_ring_pop(dn, &dones[drained])) {
            if (done_ns)
                done_ns[drained] = pump_now_ns() - t0;
            drained++;
            progress = 1;
        }
        if (progress) {
            last_progress = now;
        } else {
            /* waiting for an arrival is not a stall */
            const int waiting = pushed < n && arrival_ns && now - t0 < arrival_ns[pushed];
            if (waiting)
                last_progress = now;
            if (timeout_ms && now - last_progress > (uint64_t)timeout_ms * 1000000ull)
                return -1;
#if defined(__x86_64__)
            __asm__ volatile("pause" ::: "memory");
#endif
        }
    }
    return (int64_t)drained;
}

int64_t
rt_host_decode_pump(CommandRing *ring, const Descriptor *descs, uint32_t n, uint32_t n_sentinels,
                    CompletionRing *comp, Completion *out, uint32_t n_expected,
                    uint32_t timeout_ms)
{
    uint32_t pushed = 0, sent = 0, drained = 0;
    const uint64_t t0 = pump_now_ms();

    if (!ring || !comp || (n && !descs) || (n_expected && !out))
        return -1;
    while (drained < n_expected || pushed < n || sent < n_sentinels) {
        int progress = 0;
        /* descriptors first, then the stop records, as many as fit; one
         * tail release per batch (reference decode_batch_submit) */
        uint32_t head = rt_load_acquire_u32(&ring->cons.head);
        uint32_t tail = rt_load_relaxed_u32(&ring->prod.tail);
        uint32_t room = (uint32_t)RING_SIZE - (tail - head);
        uint32_t k = 0;
        while (k < room && (pushed < n || sent < n_sentinels)) {
            Descriptor *slot = &ring->slots[(tail + k) & (RING_SIZE - 1u)];
            if (pushed < n) {
                *slot = descs[pushed++];
            } else {
                memset(slot, 0, sizeof(*slot));
                slot->seq_id = UINT64_MAX;
                sent++;
            }
            k++;
        }
        if (k) {
            ring_commit(ring, k);
            progress = 1;
        }
        /* drain: one tail read and one head release per batch (the
         * comp_ring_poll contract, k records at a time) */
        if (drained < n_expected) {
            uint32_t chead = rt_load_relaxed_u32(&comp->cons.head);
            uint32_t ctail = rt_load_acquire_u32(&comp->prod.tail);
            uint32_t avail = ctail - chead;
            if (avail > n_expected - drained)
                avail = n_expected - drained;
            for (uint32_t i = 0; i < avail; i++)
                out[drained + i] = comp->slots[(chead + i) & (COMP_RING_SIZE - 1u)];
            if (avail) {
                rt_store_release_u32(&comp->cons.head, chead + avail);
                drained += avail;
                progress = 1;
            }
        }
        if (!progress) {
            if (timeout_ms && pump_now_ms() - t0 > timeout_ms)
                return -1;
#if defined(__x86_64__)
            __asm__ volatile("pause" ::: "memory");
#endif
        }
    }
    return (int64_t)drained;
}
