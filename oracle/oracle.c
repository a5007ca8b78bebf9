/*
 * oracle.c - CPU restatement of the reference rollout hot path.
 * TEST INFRASTRUCTURE ONLY (see oracle.h): used by tests/, smoke() and the
 * CPU-baseline leg of bench.py as the checker, never by the product.
 * Build: oracle/Makefile (gcc -O2 -fopenmp -ffp-contract=off).
 */
#include "oracle.h"

#include <float.h>
#include <math.h>
#include <stdlib.h>
#include <string.h>

/* ---------------------------------------------------------------- Philox */
/* Philox4x32-10 as published by Salmon et al. (SC'11, "Parallel random
 * numbers: as easy as 1, 2, 3"): two 32x32->64 multiplies per round with
 * multipliers 0xD2511F53 / 0xCD9E8D57, Weyl key increments 0x9E3779B9 /
 * 0xBB67AE85, ten rounds. */
void
orc_philox4x32_10(const uint32_t ctr[4], const uint32_t key[2], uint32_t out[4])
{
    uint32_t c0 = ctr[0], c1 = ctr[1], c2 = ctr[2], c3 = ctr[3];
    uint32_t k0 = key[0], k1 = key[1];
    for (int r = 0; r < 10; r++) {
        uint64_t p0 = (uint64_t)0xD2511F53u * c0;
        uint64_t p1 = (uint64_t)0xCD9E8D57u * c2;
        uint32_t hi0 = (uint32_t)(p0 >> 32), lo0 = (uint32_t)p0;
        uint32_t hi1 = (uint32_t)(p1 >> 32), lo1 = (uint32_t)p1;
        c0 = hi1 ^ c1 ^ k0;
        c1 = lo1;
        c2 = hi0 ^ c3 ^ k1;
        c3 = lo0;
        k0 += 0x9E3779B9u;
        k1 += 0xBB67AE85u;
    }
    out[0] = c0; out[1] = c1; out[2] = c2; out[3] = c3;
}

uint32_t
orc_sample_u24(uint64_t seed, uint32_t rollout_id, uint64_t step)
{
    uint32_t ctr[4] = {(uint32_t)step, (uint32_t)(step >> 32), rollout_id, 0u};
    uint32_t key[2] = {(uint32_t)seed, (uint32_t)(seed >> 32)};
    uint32_t out[4];
    orc_philox4x32_10(ctr, key, out);
    return out[0] & 0x00FFFFFFu;
}

/* ----------------------------------------------------------- conversions */
float
orc_bf16_to_f32(uint16_t b)
{
    uint32_t u = (uint32_t)b << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

uint16_t
orc_f32_to_bf16_rne(float f)
{
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7F800000u) == 0x7F800000u && (u & 0x007FFFFFu))
        return (uint16_t)((u >> 16) | 0x0040u);
    u += 0x7FFFu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

float
orc_f16_to_f32(uint16_t h)
{
    uint32_t sign = (uint32_t)(h >> 15) << 31;
    uint32_t exp = (h >> 10) & 0x1Fu;
    uint32_t man = h & 0x3FFu;
    float f;
    if (exp == 0) {
        f = ldexpf((float)man, -24);
        return sign ? -f : f;
    }
    if (exp == 31) {
        uint32_t u = sign | 0x7F800000u | (man << 13);
        memcpy(&f, &u, 4);
        return f;
    }
    {
        uint32_t u = sign | ((exp + 112u) << 23) | (man << 13);
        memcpy(&f, &u, 4);
        return f;
    }
}

uint16_t
orc_f32_to_f16_rne(float f)
{
    /* Exact for the values the tests use (normal fp16 range and zero);
     * rounds to nearest even via double arithmetic. */
    double a = fabs((double)f);
    uint16_t sign = signbit(f) ? 0x8000u : 0u;
    if (a == 0.0)
        return sign;
    if (a >= 65520.0)
        return (uint16_t)(sign | 0x7C00u);
    int e;
    (void)frexp(a, &e);               /* a = m * 2^e, m in [0.5,1) */
    int exp16 = e - 1 + 15;
    if (exp16 <= 0) {                  /* subnormal: multiple of 2^-24 */
        double q = nearbyint(a * 16777216.0);
        return (uint16_t)(sign | (uint16_t)q);
    }
    double scaled = a / ldexp(1.0, e - 11);   /* in [1024, 2048) */
    double q = nearbyint(scaled);
    if (q >= 2048.0) {
        q /= 2.0;
        exp16++;
        if (exp16 >= 31)
            return (uint16_t)(sign | 0x7C00u);
    }
    return (uint16_t)(sign | (uint16_t)(exp16 << 10) | (uint16_t)((uint32_t)q - 1024u));
}

/* ------------------------------------------------------ paged attention */
static inline uint64_t
page_off(uint64_t page, uint32_t head, uint32_t plane, uint32_t tok,
         uint32_t Hkv, uint32_t D)
{
    return ((((page * Hkv + head) * 2u + plane) * 16u + tok) * (uint64_t)D);
}

void
orc_paged_gqa_attention(const uint16_t *q, const uint16_t *arena,
                        const int32_t *page_table, const int32_t *seq_lens,
                        uint32_t B, uint32_t Hq, uint32_t Hkv, uint32_t D,
                        uint32_t max_pages, float scale, float *out, int n_threads)
{
    const uint32_t G = Hq / Hkv;
    int64_t work = (int64_t)B * Hkv;
    if (n_threads <= 0)
        n_threads = 1;
#pragma omp parallel for schedule(dynamic, 1) num_threads(n_threads)
    for (int64_t wi = 0; wi < work; wi++) {
        uint32_t b = (uint32_t)(wi / Hkv), hk = (uint32_t)(wi % Hkv);
        int32_t L = seq_lens[b];
        double *s = (double *)malloc(sizeof(double) * (size_t)(L > 0 ? L : 1));
        double *acc = (double *)malloc(sizeof(double) * D);
        for (uint32_t g = 0; g < G; g++) {
            uint32_t hq = hk * G + g;
            const uint16_t *qv = q + ((uint64_t)b * Hq + hq) * D;
            float *o = out + ((uint64_t)b * Hq + hq) * D;
            if (L <= 0) {
                for (uint32_t d = 0; d < D; d++)
                    o[d] = 0.0f;
                continue;
            }
            double m = -INFINITY;
            for (int32_t t = 0; t < L; t++) {
                int32_t pg = page_table[(uint64_t)b * max_pages + (uint32_t)t / 16u];
                const uint16_t *kv = arena + page_off((uint64_t)pg, hk, 0, (uint32_t)t % 16u, Hkv, D);
                double dot = 0.0;
                for (uint32_t d = 0; d < D; d++)
                    dot += (double)orc_bf16_to_f32(qv[d]) * (double)orc_bf16_to_f32(kv[d]);
                s[t] = dot * (double)scale;
                if (s[t] > m)
                    m = s[t];
            }
            double den = 0.0;
            for (uint32_t d = 0; d < D; d++)
                acc[d] = 0.0;
            for (int32_t t = 0; t < L; t++) {
                int32_t pg = page_table[(uint64_t)b * max_pages + (uint32_t)t / 16u];
                const uint16_t *vv = arena + page_off((uint64_t)pg, hk, 1, (uint32_t)t % 16u, Hkv, D);
                double p = exp(s[t] - m);
                den += p;
                for (uint32_t d = 0; d < D; d++)
                    acc[d] += p * (double)orc_bf16_to_f32(vv[d]);
            }
            for (uint32_t d = 0; d < D; d++)
                o[d] = (float)(acc[d] / den);
        }
        free(s);
        free(acc);
    }
}

/* ----------------------------------------------------- fixed128 (ref v0.2) */
/* Plain softmax attention of one fp32 query over the first seq_len tokens
 * of a 16 KiB fp16 block (K plane, then V plane), in the order of the
 * reference test's CPU reference (test/test_bench.cu:109-150). */
static void
fixed128_core(const float *q, const uint16_t *block_f16, uint32_t seq_len, float *out)
{
    float scores[32], probs[32];
    const uint16_t *v = block_f16 + 32u * 128u;
    const float scale = 1.0f / sqrtf(128.0f);
    float mx = -1.0e30f, den = 0.0f;
    if (seq_len > 32u)
        seq_len = 32u;
    for (uint32_t t = 0; t < seq_len; t++) {
        float dot = 0.0f;
        for (uint32_t d = 0; d < 128u; d++)
            dot += q[d] * orc_f16_to_f32(block_f16[t * 128u + d]);
        scores[t] = dot * scale;
        if (scores[t] > mx)
            mx = scores[t];
    }
    for (uint32_t t = 0; t < seq_len; t++) {
        probs[t] = expf(scores[t] - mx);
        den += probs[t];
    }
    if (den == 0.0f)
        den = 1.0f;
    for (uint32_t d = 0; d < 128u; d++)
        out[d] = 0.0f;
    for (uint32_t t = 0; t < seq_len; t++) {
        float p = probs[t] / den;
        for (uint32_t d = 0; d < 128u; d++)
            out[d] += p * orc_f16_to_f32(v[t * 128u + d]);
    }
}

void
orc_fixed128_attention(const uint16_t *q_f16, const uint16_t *block_f16,
                       uint32_t seq_len, float *out, uint32_t *token_id)
{
    float q[128];
    for (uint32_t d = 0; d < 128u; d++)
        q[d] = orc_f16_to_f32(q_f16[d]);
    fixed128_core(q, block_f16, seq_len, out);
    /* test/test_bench.cu:151-155: lowest index wins ties */
    *token_id = 0;
    for (uint32_t d = 1; d < 128u; d++)
        if (out[d] > out[*token_id])
            *token_id = d;
}

/* Reference cu/attention_decode.cu:16-28 (decode_synth_query_component). */
float
orc_decode_synth_q(uint64_t seq_id, uint64_t cookie, const uint64_t *rng4, uint32_t idx)
{
    uint64_t seed = seq_id ^ cookie ^ ((uint64_t)(idx + 1u) * 0x9e3779b97f4a7c15ull);
    if (rng4)
        seed ^= rng4[idx & 3u];
    const uint32_t bits = (uint32_t)(seed ^ (seed >> 32));
    const int centered = (int)(bits & 0xFFu) - 127;
    return (float)centered / 127.0f;
}

/* Reference cu/attention_decode.cu:171-194: each lane keeps the first
 * strict maximum of d = lane, lane+32, ...; lane 0 then keeps the first
 * strict maximum over lanes 0..31.  Equivalent: scan d in (d mod 32,
 * d / 32) order with a strict '>' from -inf; nothing above -inf -> 0. */
static uint32_t
kernel_argmax(const float *o)
{
    float best = -INFINITY;
    uint32_t tok = 0;
    for (uint32_t lane = 0; lane < 32u; lane++)
        for (uint32_t j = 0; j < 4u; j++) {
            const uint32_t d = lane + 32u * j;
            if (o[d] > best) {
                best = o[d];
                tok = d;
            }
        }
    return tok;
}

uint32_t
orc_decode_steps(const Descriptor *descs, uint32_t n, const uint8_t *arena, uint64_t block_size,
                 uint64_t n_blocks, const uint64_t *rng4, const uint16_t *q_buf,
                 uint32_t io_slots, float *o_rows, Completion *comps)
{
    uint32_t bad = 0;
    for (uint32_t i = 0; i < n; i++) {
        const Descriptor *d = &descs[i];
        Completion c;
        float o[128], q[128];
        /* cu/worker.cu:34-39 */
        const uint32_t slot = io_slots == 0u ? 0u : (d->output_token_offset & (io_slots - 1u));
        uint32_t seq_len = d->num_kv_blocks == 0u ? 1u : d->num_kv_blocks;
        if (seq_len > 32u)
            seq_len = 32u;
        c.seq_id = d->seq_id;
        c.kv_block_offset = d->kv_block_offset;
        c.reward_cookie = d->reward_cookie;
        if ((uint64_t)d->kv_block_offset >= n_blocks) {
            /* out-of-range block: flagged record, no output row */
            c.token_id = UINT32_MAX;
            c.cycles_taken = 0;
            bad++;
            if (o_rows)
                memset(o_rows + (size_t)i * 128u, 0, 128u * sizeof(float));
        } else {
            for (uint32_t k = 0; k < 128u; k++)
                q[k] = q_buf ? orc_f16_to_f32(q_buf[(size_t)slot * 128u + k])
                             : orc_decode_synth_q(d->seq_id, d->reward_cookie, rng4, k);
            fixed128_core(q, (const uint16_t *)(arena + (uint64_t)d->kv_block_offset * block_size),
                          seq_len, o);
            c.token_id = kernel_argmax(o);
            /* cu/attention_decode.cu:196-201 */
            c.cycles_taken = (uint64_t)((seq_len + 15u) / 16u) * 128u * 24u;
            if (o_rows)
                memcpy(o_rows + (size_t)i * 128u, o, sizeof(o));
        }
        comps[i] = c;
    }
    return bad;
}

/* ---------------------------------------------------------- worker sim */
/* One token per iteration, exactly as reference src/hw_worker_sim.c:39-52. */
uint32_t
orc_worker_sim_stream(const hw_desc_t *in, uint32_t n, hw_desc_t *done,
                      uint64_t *decoded_tokens)
{
    uint32_t nd = 0;
    uint64_t tokens = 0;
    for (uint32_t i = 0; i < n; i++) {
        hw_desc_t d = in[i];
        if (d.opcode == DESC_OP_STOP)
            break;
        if (d.opcode != DESC_OP_DECODE)
            continue;
        while (d.seq_len < d.max_tokens) {
            d.seq_len++;
            tokens++;
            if (d.seq_len >= d.max_tokens) {
                d.flags |= DESC_FLAG_DONE;
                break;
            }
            if ((d.seq_len & 31u) == 0u) {
                d.flags |= DESC_FLAG_NEEDS_REWARD;
                break;
            }
        }
        done[nd++] = d;
    }
    *decoded_tokens = tokens;
    return nd;
}

void
orc_submit_desc(uint32_t gpu_group_id, uint32_t kv_arena_id, uint32_t rollout_id,
                uint64_t kv_offset, uint64_t delta_offset, uint32_t prefix_id,
                uint32_t seq_len, uint32_t max_tokens, hw_desc_t *o)
{
    memset(o, 0, sizeof(*o));
    o->opcode = DESC_OP_DECODE;
    o->flags = prefix_id ? DESC_FLAG_COW_PREFIX : 0u;
    o->rollout_id = rollout_id;
    o->kv_arena_id = kv_arena_id;
    o->prefix_id = prefix_id;
    o->kv_offset = kv_offset;
    o->delta_offset = delta_offset;
    o->seq_len = seq_len;
    o->max_tokens = max_tokens;
    o->reward_model_id = 0;
    o->reserved0 = gpu_group_id;
    o->user_data = rollout_id;
    o->checksum_or_cookie = kv_offset ^ delta_offset ^ ((uint64_t)rollout_id << 32);
}

/* -------------------------------------------------------------- sampler */
uint32_t
orc_sample_row(const float *logits, uint32_t V, float temperature, uint32_t top_k,
               float top_p, uint32_t u24, int fma_cum, float *l)
{
    memcpy(l, logits, sizeof(float) * V);
    if (temperature > 0.0f) {
        float inv = 1.0f / temperature;
        for (uint32_t i = 0; i < V; i++)
            l[i] *= inv;
    }
    if (top_k > 0u && top_k < V) {
        float th[256];
        uint32_t nk = top_k < 256u ? top_k : 256u;
        for (uint32_t j = 0; j < nk; j++)
            th[j] = -FLT_MAX;
        for (uint32_t i = 0; i < V; i++) {
            float v = l[i];
            for (uint32_t j = 0; j < nk; j++) {
                if (v > th[j]) {
                    for (uint32_t k = nk - 1u; k > j; k--)
                        th[k] = th[k - 1u];
                    th[j] = v;
                    break;
                }
            }
        }
        float cutoff = th[nk - 1u];
        for (uint32_t i = 0; i < V; i++)
            if (l[i] < cutoff)
                l[i] = -FLT_MAX;
    }
    float r = (float)(u24 & 0x00FFFFFFu) / 16777216.0f;
    float mx = -FLT_MAX, sum = 0.0f, cum = 0.0f;
    for (uint32_t i = 0; i < V; i++)
        if (l[i] > mx)
            mx = l[i];
    if (top_p > 0.0f && top_p < 1.0f) {
        for (uint32_t i = 0; i < V; i++)
            sum += expf(l[i] - mx);
        float inv = 1.0f / sum;
        for (uint32_t i = 0; i < V; i++) {
            float e = expf(l[i] - mx);
            cum = fma_cum ? fmaf(e, inv, cum) : cum + e * inv;
            if (cum >= r)
                return i;
        }
        return V - 1u;
    }
    for (uint32_t i = 0; i < V; i++) {
        l[i] = expf(l[i] - mx);
        sum += l[i];
    }
    for (uint32_t i = 0; i < V; i++) {
        cum += l[i] / sum;
        if (cum >= r)
            return i;
    }
    return V - 1u;
}

/* ------------------------------------------------------------ scheduler */
/* Lowest free slot (reference find_free_slot, cu/gpu_scheduler.cu:4-16),
 * restricted to slots below max_slots (the reference always has 256). */
static int
sched_take_slot(GpuRolloutState *st, uint32_t max_slots)
{
    for (int w = 0; w < (GPU_MAX_ROLLOUTS + 63) / 64; w++) {
        uint64_t free_bits = ~st->bitmap[w];
        const uint32_t lo = (uint32_t)w * 64u;
        if (lo >= max_slots)
            break;
        if (max_slots - lo < 64u)
            free_bits &= (1ull << (max_slots - lo)) - 1ull;
        if (free_bits) {
            int b = __builtin_ctzll(free_bits);
            st->bitmap[w] |= 1ull << b;
            return w * 64 + b;
        }
    }
    return -1;
}

uint32_t
orc_scheduler_run(const RolloutRequest *reqs, uint32_t n_reqs,
                  const uint32_t *arrival_pass, uint32_t max_admit,
                  int drop_when_full, uint32_t max_passes,
                  RolloutDone *dones, uint32_t *done_pass,
                  GpuRolloutState *st, uint32_t *passes_run, uint32_t *admit_pass,
                  uint32_t max_slots)
{
    if (max_slots == 0 || max_slots > GPU_MAX_ROLLOUTS)
        max_slots = GPU_MAX_ROLLOUTS;
    uint32_t next = 0, nd = 0, pass = 0, active = 0;
    memset(st, 0, sizeof(*st));
    if (admit_pass)
        for (uint32_t i = 0; i < n_reqs; i++)
            admit_pass[i] = UINT32_MAX;
    for (pass = 0; pass < max_passes; pass++) {
        int stop = 0;
        for (uint32_t a = 0; a < max_admit; a++) {
            if (next >= n_reqs || (arrival_pass && arrival_pass[next] > pass))
                break;
            RolloutRequest rq = reqs[next];
            if (rq.request_id == UINT64_MAX) {
                next++;
                stop = 1;
                break;
            }
            int s = sched_take_slot(st, max_slots);
            if (s < 0) {
                if (drop_when_full) {
                    next++;
                    continue;
                }
                break;
            }
            if (admit_pass)
                admit_pass[next] = pass;
            next++;
            GpuRolloutSlot *rs = &st->slots[s];
            rs->active = 1;
            rs->request_id = (uint32_t)(rq.request_id & 0xFFFFFFFFu);
            rs->tokens_generated = 0;
            rs->max_tokens = rq.max_tokens;
            rs->kv_blocks = rq.kv_blocks;
            rs->rng_state[0] = rq.rng_seed;
            rs->rng_state[1] = rq.rng_seed ^ 0x9e3779b97f4a7c15ULL;
            rs->rng_state[2] = (rq.rng_seed << 17) ^ 0x3c6ef372fe94f82aULL;
            rs->rng_state[3] = ~rq.rng_seed;
            rs->temperature = rq.temperature;
            rs->top_k = rq.top_k;
            rs->top_p = rq.top_p;
            active++;
        }
        if (stop) {
            pass++;
            break;
        }
        for (int s = 0; s < GPU_MAX_ROLLOUTS; s++) {
            GpuRolloutSlot *rs = &st->slots[s];
            if (!rs->active)
                continue;
            if (rs->tokens_generated >= rs->max_tokens) {
                rs->active = 0;
                RolloutDone d;
                d.request_id = rs->request_id;
                d.rollout_id = (uint32_t)s;
                d.tokens_generated = rs->tokens_generated;
                d.reward = (float)(rs->tokens_generated & 0xFFu) / 255.0f;
                d.status = 0;
                if (dones)
                    dones[nd] = d;
                if (done_pass)
                    done_pass[nd] = pass;
                nd++;
                st->bitmap[s / 64] &= ~(1ull << (s % 64));
                active--;
                continue;
            }
            rs->tokens_generated++;
        }
        if (next >= n_reqs && active == 0) {
            pass++;
            break;
        }
    }
    if (passes_run)
        *passes_run = pass;
    return nd;
}

/* Reward of a finished rollout in the Philox reward mode:
 * U(0,1) = (word0 >> 8) / 2^24, key = seed, counter = {request low 32, 0,
 * 0x52455744, 0}. */
float
orc_reward_u01(uint64_t seed, uint32_t request_lo)
{
    uint32_t ctr[4] = {request_lo, 0u, 0x52455744u, 0u};
    uint32_t key[2] = {(uint32_t)seed, (uint32_t)(seed >> 32)};
    uint32_t out[4];
    orc_philox4x32_10(ctr, key, out);
    return (float)(out[0] >> 8) * (1.0f / 16777216.0f);
}

/* ----------------------------------------------------------- advantages */
void
orc_grpo_advantages(const float *r, uint32_t n, uint32_t G, float eps, float *adv)
{
    for (uint32_t g0 = 0; g0 + G <= n; g0 += G) {
        float sum = 0.0f, var = 0.0f;
        for (uint32_t i = 0; i < G; i++)
            sum += r[g0 + i];
        float mean = sum / (float)G;
        for (uint32_t i = 0; i < G; i++) {
            float dlt = r[g0 + i] - mean;
            float sq = dlt * dlt;
            var += sq;
        }
        float sd = sqrtf(var / (float)G);
        float den = sd + eps;
        for (uint32_t i = 0; i < G; i++)
            adv[g0 + i] = (r[g0 + i] - mean) / den;
    }
}
