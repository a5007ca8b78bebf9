/*
 * abi_caller.c - a caller of the rollout runtime's C API, written only
 * against the public headers.  TEST INFRASTRUCTURE ONLY.
 *
 * oracle/Makefile compiles this one source twice: once against the
 * reference's headers and C sources (oracle/_ref/libabi_ref.so, built from
 * the read-only reference tree) and once against this repository's headers
 * and librlrt_b200.so (oracle/_build/libabi_mine.so).  The parity tests call
 * the same hx_* function in both builds and require identical bytes out,
 * which is what "drop-in" means for a C caller.  The scripted sequences
 * follow the reference's own tests (test/test_hw_ring.c, test/test_smoke.c,
 * test/test_bench.cu:512-797).
 */
#define _GNU_SOURCE
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

#include "hw_desc.h"
#include "hw_ring.h"
#include "hw_worker_sim.h"
#include "infer_submit.h"
#include "mmio.h"
#include "descriptor.h"
#include "completion.h"
#include "ring.h"
#include "decode_batch.h"
#include "request.h"
#include "reward.h"
#include "kv_prefix.h"
#include "arena.h"

static inline void
hx_relax(void)
{
#if defined(__x86_64__)
    __asm__ volatile("pause" ::: "memory");
#endif
}

static double
hx_now(void)
{
    struct timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return (double)ts.tv_sec + 1e-9 * (double)ts.tv_nsec;
}

/* ---- C1 workload: splitmix64-seeded xoshiro256** (Blackman & Vigna) ---- */
static uint64_t
hx_splitmix64(uint64_t *x)
{
    uint64_t z = (*x += 0x9e3779b97f4a7c15ULL);
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ULL;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebULL;
    return z ^ (z >> 31);
}

static uint64_t
hx_rotl(uint64_t x, int k)
{
    return (x << k) | (x >> (64 - k));
}

static uint64_t
hx_xoshiro(uint64_t s[4])
{
    uint64_t r = hx_rotl(s[1] * 5u, 7) * 9u;
    uint64_t t = s[1] << 17;
    s[2] ^= s[0];
    s[3] ^= s[1];
    s[1] ^= s[2];
    s[0] ^= s[3];
    s[2] ^= t;
    s[3] = hx_rotl(s[3], 45);
    return r;
}

/* Uniform integer in [0, n) by multiply-shift of the high 32 bits. */
static uint32_t
hx_below(uint64_t s[4], uint32_t n)
{
    return (uint32_t)(((hx_xoshiro(s) >> 32) * (uint64_t)n) >> 32);
}

void
hx_gen_c1(uint64_t seed, uint32_t n, uint32_t max_tokens, hw_desc_t *out)
{
    uint64_t sm = seed, s[4];
    for (int i = 0; i < 4; i++)
        s[i] = hx_splitmix64(&sm);
    for (uint32_t i = 0; i < n; i++) {
        hw_desc_t d;
        memset(&d, 0, sizeof(d));
        d.opcode = DESC_OP_DECODE;
        d.rollout_id = hx_below(s, 256u);
        d.seq_len = hx_below(s, 2048u);
        d.kv_offset = hx_below(s, 4096u);
        d.max_tokens = max_tokens;
        out[i] = d;
    }
}

/* ---- C1 run: producer (this thread) -> cmdq -> hw_worker_sim -> doneq ---- */
typedef struct {
    hw_worker_sim_t *w;
} hx_thread_arg;

static void *
hx_worker_main(void *p)
{
    hw_worker_sim_run(((hx_thread_arg *)p)->w);
    return NULL;
}

/* Runs n descriptors through the worker with at most depth_cap in flight;
 * done records are copied to out in doneq order.  Returns 0 on success. */
int
hx_run_c1(const hw_desc_t *in, uint32_t n, uint32_t depth_cap, uint32_t doorbell_batch,
          hw_desc_t *out, uint32_t *n_out, uint64_t *tokens, uint64_t *completions,
          double *seconds)
{
    hw_ring_t *cmdq = hw_ring_create();
    hw_ring_t *doneq = hw_ring_create();
    volatile uint32_t stop = 0, doorbell = 0;
    hw_worker_sim_t w;
    hx_thread_arg arg;
    pthread_t th;
    uint32_t expected = 0, submitted = 0, completed = 0;
    double t0, t1;

    if (!cmdq || !doneq)
        return -1;
    for (uint32_t i = 0; i < n; i++)
        expected += (in[i].opcode == DESC_OP_DECODE);
    memset(&w, 0, sizeof(w));
    w.cmdq = cmdq;
    w.doneq = doneq;
    w.stop = &stop;
    arg.w = &w;
    if (pthread_create(&th, NULL, hx_worker_main, &arg) != 0)
        return -1;

    t0 = hx_now();
    for (uint32_t i = 0; i < n; i++) {
        hw_desc_t d;
        while (submitted - completed >= depth_cap || hw_ring_full(cmdq)) {
            while (hw_ring_pop(doneq, &d) == 0)
                out[completed++] = d;
            hx_relax();
        }
        d = in[i];
        while (hw_ring_push(cmdq, &d) != 0)
            hx_relax();
        if (in[i].opcode == DESC_OP_DECODE)
            submitted++;
        if (((i + 1u) % doorbell_batch) == 0u || i + 1u == n)
            mmio_write32(&doorbell, hw_ring_load_acquire(&cmdq->tail));
    }
    while (completed < expected) {
        hw_desc_t d;
        if (hw_ring_pop(doneq, &d) == 0)
            out[completed++] = d;
        else
            hx_relax();
    }
    t1 = hx_now();

    {
        hw_desc_t s;
        memset(&s, 0, sizeof(s));
        s.opcode = DESC_OP_STOP;
        while (hw_ring_push(cmdq, &s) != 0)
            hx_relax();
    }
    pthread_join(th, NULL);
    *n_out = completed;
    *tokens = w.decoded_tokens;
    *completions = w.completions;
    *seconds = t1 - t0;
    hw_ring_destroy(cmdq);
    hw_ring_destroy(doneq);
    return 0;
}

/* ---- host batching (host side): decode_batch_push /
 * decode_batch_submit windows of `window` descriptors into a CommandRing
 * (reference src/decode_batch.c:12-42) on this thread, ring_consume of every
 * record on a second thread into out[] (ring order).  Returns 0 and the
 * seconds from the first push to the last record consumed. ---- */
typedef struct {
    CommandRing *ring;
    Descriptor *out;
    uint32_t n;
} hx_consumer_arg;

static void *
hx_consumer_main(void *p)
{
    hx_consumer_arg *a = (hx_consumer_arg *)p;
    uint32_t got = 0;
    while (got < a->n) {
        if (ring_consume(a->ring, &a->out[got]))
            got++;
        else
            hx_relax();
    }
    return NULL;
}

int
hx_run_decode_batch(const Descriptor *in, uint32_t n, uint32_t window, Descriptor *out,
                    double *seconds)
{
    CommandRing *ring = ring_create();
    DecodeDispatchBatch batch;
    hx_consumer_arg arg;
    pthread_t th;
    double t0, t1;

    if (!ring || window == 0 || window > DECODE_DESCRIPTOR_BATCH_LIMIT)
        return -1;
    arg.ring = ring;
    arg.out = out;
    arg.n = n;
    if (pthread_create(&th, NULL, hx_consumer_main, &arg) != 0)
        return -1;
    t0 = hx_now();
    for (uint32_t i = 0; i < n; i += window) {
        const uint32_t k = n - i < window ? n - i : window;
        decode_batch_reset(&batch);
        for (uint32_t j = 0; j < k; j++)
            decode_batch_push(&batch, &in[i + j]);
        while (decode_batch_submit(ring, &batch) != 0)   /* ring full: wait for the consumer */
            hx_relax();
    }
    pthread_join(th, NULL);
    t1 = hx_now();
    *seconds = t1 - t0;
    ring_destroy(ring);
    return 0;
}

/* ---- known-answer scripts (reference test/test_hw_ring.c:98-154) ---- */
int
hx_kat_submit(uint32_t gpu_group, uint32_t arena_id, uint32_t rollout, uint64_t kv,
              uint64_t delta, uint32_t prefix, uint32_t seq, uint32_t max_tokens,
              uint32_t *doorbell_out, hw_desc_t *desc_out)
{
    hw_ring_t *cmdq = hw_ring_create(), *doneq = hw_ring_create();
    volatile uint32_t doorbell = 0;
    infer_hw_ctx_t ctx;
    int rc;
    memset(&ctx, 0, sizeof(ctx));
    ctx.cmdq = cmdq;
    ctx.doneq = doneq;
    ctx.doorbell = &doorbell;
    ctx.gpu_group_id = gpu_group;
    ctx.kv_arena_id = arena_id;
    rc = infer_submit_decode(&ctx, rollout, kv, delta, prefix, seq, max_tokens);
    *doorbell_out = doorbell;
    if (rc == 0 && hw_ring_pop(cmdq, desc_out) != 0)
        rc = -2;
    hw_ring_destroy(cmdq);
    hw_ring_destroy(doneq);
    return rc;
}

/* Error paths of the submit API: NULL ctx / cmdq / doorbell and full ring.
 * Writes the four return codes. */
void
hx_kat_submit_errors(int rc[4])
{
    hw_ring_t *cmdq = hw_ring_create();
    volatile uint32_t doorbell = 0;
    infer_hw_ctx_t ctx;
    hw_desc_t d;
    memset(&ctx, 0, sizeof(ctx));
    rc[0] = infer_submit_decode(NULL, 1, 0, 0, 0, 0, 1);
    rc[1] = infer_submit_decode(&ctx, 1, 0, 0, 0, 0, 1);
    ctx.cmdq = cmdq;
    rc[2] = infer_submit_decode(&ctx, 1, 0, 0, 0, 0, 1);
    ctx.doorbell = &doorbell;
    memset(&d, 0, sizeof(d));
    for (uint32_t i = 0; i < HW_RING_SIZE; i++)
        hw_ring_push(cmdq, &d);
    rc[3] = infer_submit_decode(&ctx, 1, 0, 0, 0, 0, 1);
    hw_ring_destroy(cmdq);
}

/* Ring invariants of reference test/test_hw_ring.c:20-154.  Returns a
 * bitmask of the checks that held (all = 0x3F). */
uint32_t
hx_kat_hw_ring(void)
{
    uint32_t ok = 0;
    hw_ring_t *r = hw_ring_create();
    hw_desc_t d, o;
    int good = 1;
    memset(&d, 0, sizeof(d));
    if (hw_ring_empty(r))
        ok |= 1u;
    for (uint32_t i = 0; i < HW_RING_SIZE; i++) {
        d.rollout_id = i;
        good &= hw_ring_push(r, &d) == 0;
    }
    if (good && hw_ring_full(r) && hw_ring_push(r, &d) == -1)
        ok |= 2u;
    for (uint32_t i = 0; i < HW_RING_SIZE / 2u; i++)
        good &= hw_ring_pop(r, &o) == 0 && o.rollout_id == i;
    for (uint32_t i = 0; i < HW_RING_SIZE / 2u; i++) {
        d.rollout_id = 100000u + i;
        good &= hw_ring_push(r, &d) == 0;
    }
    for (uint32_t i = HW_RING_SIZE / 2u; i < HW_RING_SIZE; i++)
        good &= hw_ring_pop(r, &o) == 0 && o.rollout_id == i;
    for (uint32_t i = 0; i < HW_RING_SIZE / 2u; i++)
        good &= hw_ring_pop(r, &o) == 0 && o.rollout_id == 100000u + i;
    if (good)
        ok |= 4u;
    if (hw_ring_empty(r) && hw_ring_pop(r, &o) == -1)
        ok |= 8u;
    hw_ring_reset(r);
    if (hw_ring_empty(r) && r->head == 0 && r->tail == 0)
        ok |= 16u;
    if (sizeof(hw_desc_t) == 64 && sizeof(hw_ring_t) == 128 + 64ull * HW_RING_SIZE)
        ok |= 32u;
    hw_ring_destroy(r);
    return ok;
}

/* Worker-sim single descriptor (reference test/test_hw_ring.c:168-217). */
int
hx_kat_worker(const hw_desc_t *in, hw_desc_t *out, uint64_t *tokens, uint64_t *completions)
{
    uint32_t n_out = 0;
    double secs;
    return hx_run_c1(in, 1, 1, 1, out, &n_out, tokens, completions, &secs) == 0 && n_out == 1 ? 0 : -1;
}

/* CommandRing + CompletionRing + decode batching (reference
 * test/test_smoke.c:10-199, 286-322).  Writes a transcript of return values
 * into log (capacity >= 64) and returns the number of entries. */
uint32_t
hx_script_command_ring(int64_t *log, Descriptor *batch_out)
{
    uint32_t n = 0;
    CommandRing *ring = ring_create();
    CompletionRing *cr = comp_ring_create();
    Descriptor d;
    Completion c;
    DecodeDispatchBatch batch;

    memset(&d, 0, sizeof(d));
    log[n++] = ring_consume(ring, &d);                       /* empty -> 0 */
    for (uint32_t i = 0; i < RING_SIZE; i++) {
        uint32_t pos = ring_acquire(ring, 1);
        if (pos == UINT32_MAX)
            break;
        ring->slots[pos].seq_id = i;
        ring_commit(ring, 1);
    }
    log[n++] = ring->prod.tail;                              /* 4096 */
    log[n++] = (int64_t)ring_acquire(ring, 1);               /* full -> UINT32_MAX */
    log[n++] = ring_consume(ring, &d);                       /* 1 */
    log[n++] = (int64_t)d.seq_id;                            /* 0 */
    log[n++] = (int64_t)ring_acquire(ring, 1);               /* position 0 */
    log[n++] = (int64_t)ring_acquire(ring, 2);               /* UINT32_MAX */
    for (uint32_t i = 1; i < RING_SIZE; i++)
        ring_consume(ring, &d);
    log[n++] = (int64_t)d.seq_id;                            /* 4095 */
    log[n++] = ring_consume(ring, &d);                       /* 0 */
    log[n++] = (int64_t)ring_acquire(ring, RING_SIZE);       /* wrapped position */

    memset(&c, 0, sizeof(c));
    c.seq_id = 1;
    c.token_id = 7;
    c.reward_cookie = 9;
    c.cycles_taken = 11;
    for (uint32_t i = 0; i < COMP_RING_SIZE; i++)
        comp_ring_push(cr, &c);
    log[n++] = comp_ring_push(cr, &c);                       /* -1 */
    log[n++] = cr->overflow.value;                           /* 1 */
    log[n++] = comp_ring_poll(cr, &c);                       /* 1 */
    log[n++] = comp_ring_push(cr, &c);                       /* 0 */
    log[n++] = (int64_t)c.cycles_taken;                      /* 11 */

    /* decode batching: three descriptors, then a 33rd push fails */
    ring_destroy(ring);
    ring = ring_create();
    decode_batch_reset(&batch);
    memset(&d, 0, sizeof(d));
    for (uint32_t i = 0; i < 3; i++) {
        d.seq_id = 11u + i;
        d.output_token_offset = 3u + i;
        log[n++] = decode_batch_push(&batch, &d);
    }
    log[n++] = decode_batch_submit(ring, &batch);
    log[n++] = ring->prod.tail;
    for (uint32_t i = 0; i < 3; i++)
        log[n++] = ring_consume(ring, &batch_out[i]);
    decode_batch_reset(&batch);
    log[n++] = decode_batch_submit(ring, &batch);            /* empty -> -1 */
    for (uint32_t i = 0; i < DECODE_DESCRIPTOR_BATCH_LIMIT; i++)
        decode_batch_push(&batch, &d);
    log[n++] = decode_batch_push(&batch, &d);                /* -1 */
    {
        DecodeBatchContract k = decode_batch_contract(&batch_out[2]);
        log[n++] = k.batch_size;
        log[n++] = k.batch_index;
        k = decode_batch_contract(NULL);
        log[n++] = k.batch_size;
    }
    ring_destroy(ring);
    comp_ring_destroy(cr);
    return n;
}

/* RequestRing / DoneRing (reference test/test_smoke.c:183-199 and the
 * request ring contract).  Rings are plain host structs here. */
uint32_t
hx_script_request_ring(int64_t *log, RolloutRequest *req_out, RolloutDone *done_out)
{
    uint32_t n = 0;
    RequestRing *rq = (RequestRing *)calloc(1, sizeof(RequestRing));
    DoneRing *dn = (DoneRing *)calloc(1, sizeof(DoneRing));
    RolloutRequest r;
    RolloutDone d;
    memset(&r, 0, sizeof(r));
    for (uint32_t i = 0; i < REQUEST_RING_SIZE; i++) {
        uint32_t pos = req_ring_acquire(rq);
        if (pos == UINT32_MAX)
            break;
        r.request_id = 1000u + i;
        r.max_tokens = i;
        r.top_p = 0.5f;
        rq->slots[pos] = r;
        req_ring_commit(rq);
    }
    log[n++] = rq->prod.tail;
    log[n++] = (int64_t)req_ring_acquire(rq);
    log[n++] = req_ring_consume(rq, req_out);
    log[n++] = (int64_t)req_ring_acquire(rq);
    d.request_id = 1;
    d.rollout_id = 2;
    d.tokens_generated = 3;
    d.reward = 0.5f;
    d.status = 0;
    log[n] = 0;
    for (uint32_t i = 0; i < REQUEST_RING_SIZE; i++)
        log[n] += done_ring_push(dn, &d);
    n++;
    log[n++] = done_ring_push(dn, &d);
    log[n++] = dn->overflow.value;
    log[n++] = done_ring_pop(dn, done_out);
    log[n++] = done_ring_push(dn, &d);
    free(rq);
    free(dn);
    return n;
}

/* kv_prefix table (reference test/test_bench.cu:760-797 plus the edge
 * cases of src/kv_prefix.c). */
uint32_t
hx_script_kv_prefix(int64_t *log)
{
    uint32_t n = 0, pid = 0, pid2 = 0, bid = 0, bid2 = 0;
    KVPrefixTable *t = (KVPrefixTable *)malloc(sizeof(KVPrefixTable));
    KVPrefix *p;
    kv_prefix_table_init(t);
    log[n++] = kv_prefix_register(t, 0x1000, 64, 4, &pid);
    log[n++] = pid;
    p = kv_prefix_get(t, pid);
    log[n++] = p->refcnt;
    log[n++] = p->token_len;
    log[n++] = kv_prefix_acquire(t, pid);
    log[n++] = p->refcnt;
    log[n++] = kv_prefix_release(t, pid);
    log[n++] = p->refcnt;
    log[n++] = kv_prefix_release(t, pid);                    /* last ref: freed */
    log[n++] = p->kv_block_offset;                           /* -1 */
    log[n++] = kv_prefix_release(t, pid);                    /* -1: refcnt 0 */
    log[n++] = kv_prefix_acquire(t, pid);                    /* -1 */
    log[n++] = kv_prefix_acquire(t, MAX_PREFIXES);           /* -1 */
    log[n++] = kv_prefix_get(t, MAX_PREFIXES) == NULL;
    log[n++] = kv_prefix_register(t, 0x4000, 32, 2, &pid);   /* reuses id */
    log[n++] = pid;
    log[n++] = kv_prefix_register(t, 0x8000, 48, 3, &pid2);
    log[n++] = pid2;
    log[n++] = kv_branch_alloc(t, 7, pid, 0x2000, 16, 1, &bid);
    log[n++] = bid;
    log[n++] = kv_prefix_get(t, pid)->refcnt;                /* 2 */
    log[n++] = kv_branch_total_offset(t, bid);               /* 0x4000 */
    log[n++] = kv_branch_alloc(t, 8, MAX_PREFIXES + 5u, 0x3000, 8, 1, &bid2);
    log[n++] = bid2;
    log[n++] = kv_branch_total_offset(t, bid2);              /* delta 0x3000 */
    log[n++] = kv_branch_free(t, bid);
    log[n++] = kv_branch_get(t, bid)->rollout_id == UINT32_MAX;
    log[n++] = kv_prefix_get(t, pid)->refcnt;                /* 1 */
    log[n++] = kv_branch_free(t, MAX_BRANCHES);              /* -1 */
    log[n++] = kv_branch_get(t, MAX_BRANCHES) == NULL;
    log[n++] = kv_branch_total_offset(t, MAX_BRANCHES);      /* -1 */
    log[n++] = kv_prefix_release(t, pid);
    log[n++] = kv_branch_total_offset(t, bid);               /* released prefix: -1 */
    for (uint32_t i = 0; i < MAX_PREFIXES + 2u; i++) {
        uint32_t id;
        if (kv_prefix_register(t, (int64_t)i, 1, 1, &id) != 0) {
            log[n++] = i;                                     /* first failure index */
            break;
        }
    }
    log[n++] = (int64_t)sizeof(KVPrefix);
    log[n++] = (int64_t)sizeof(KVBranch);
    free(t);
    return n;
}

/* Reward ring (reference test/test_bench.cu:731-757). */
uint32_t
hx_script_reward(int64_t *log, float *score_out)
{
    uint32_t n = 0;
    RewardRing *rr = (RewardRing *)malloc(sizeof(RewardRing));
    RewardDesc d, got;
    reward_ring_init(rr);
    memset(&d, 0, sizeof(d));
    d.rollout_id = 1;
    d.token_count = 128;
    log[n++] = reward_push(rr, &d);
    log[n++] = reward_pop(rr, &got);
    log[n++] = got.rollout_id;
    log[n++] = got.token_count;
    log[n++] = reward_pop(rr, &got);
    for (uint32_t i = 0; i < REWARD_RING_SIZE; i++)
        reward_push(rr, &d);
    log[n++] = reward_push(rr, &d);
    for (uint32_t i = 0; i < 600; i++)
        score_out[i] = reward_score_mock(NULL, i);
    free(rr);
    return n;
}

/* Arena bitmap order on a struct that is not backed by memory (the
 * allocator itself never dereferences base). */
uint32_t
hx_script_arena_bitmap(int64_t *log, uint32_t n_blocks)
{
    uint32_t n = 0;
    KVArena *a = (KVArena *)calloc(1, sizeof(KVArena));
    a->capacity = (size_t)n_blocks * 4096u;
    a->block_size = 4096u;
    for (uint32_t i = 0; i < 70; i++)
        log[n++] = arena_acquire(a);
    arena_release(a, 3);
    arena_release(a, 64);
    arena_release(a, -1);
    log[n++] = arena_acquire(a);
    log[n++] = arena_acquire(a);
    log[n++] = arena_acquire(a);
    free(a);
    return n;
}
