/*
 * oracle.h - CPU restatement of the reference's rollout hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the checker the parity tests,
 * __graft_entry__.smoke() and bench.py's CPU-baseline leg compare the CUDA
 * product against.  Nothing in the product links, loads or calls it.
 *
 * Each function names the reference file:line it restates.  Parity pins:
 *   - worker-sim stream, submit, decode batching, rings, kv_prefix, reward:
 *     checked against the reference's own C sources compiled unmodified into
 *     oracle/_ref (oracle/Makefile) and against the reference tests' known
 *     answers (test/test_hw_ring.c, test/test_smoke.c).
 *   - fixed128 attention: reference test/test_bench.cu:91-155 known-answer
 *     inputs; GPU kernel of the reference run through oracle/_ref on a B200.
 *   - sampler: reference cu/sample.cu:40-123 semantics with an injected
 *     24-bit uniform; bit-exact pin GPU-vs-GPU against the reference
 *     sample_token compiled into oracle/_ref (CPU expf is tolerance-only).
 *   - paged GQA attention, Philox, scheduler loop, GRPO advantages: the
 *     reference has no test for these (paging/GQA/Philox/advantages do not
 *     exist there); the restatement here is the specification
 *     ("parity unpinned" for those rows beyond Philox's published
 *     known-answer vectors).
 */
#pragma once
#include <stddef.h>
#include <stdint.h>
#include "hw_desc.h"
#include "request.h"
#include "descriptor.h"
#include "completion.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Philox4x32-10 (Salmon, Moraes, Dror, Shaw, SC'11). */
void orc_philox4x32_10(const uint32_t ctr[4], const uint32_t key[2], uint32_t out[4]);

float orc_bf16_to_f32(uint16_t b);
uint16_t orc_f32_to_bf16_rne(float f);

/* Paged GQA decode attention; q bf16 [B][Hq][D], arena bf16 pages in the
 * layout of kv_layout.h, out fp32 [B][Hq][D].  Accumulates in double.
 * Sequences of length 0 produce zeros. */
void orc_paged_gqa_attention(const uint16_t *q, const uint16_t *arena,
                             const int32_t *page_table, const int32_t *seq_lens,
                             uint32_t B, uint32_t Hq, uint32_t Hkv, uint32_t D,
                             uint32_t max_pages, float scale, float *out,
                             int n_threads);

/* Reference test/test_bench.cu:109-155 (CPU reference of the fixed128
 * step): fp16 q[128], one 16 KiB block (K plane then V plane), plain
 * softmax, argmax with the lowest index winning ties. */
void orc_fixed128_attention(const uint16_t *q_f16, const uint16_t *block_f16,
                            uint32_t seq_len, float *out, uint32_t *token_id);
float orc_f16_to_f32(uint16_t h);

/* Reference cu/attention_decode.cu:16-28: component idx of the synthesized
 * query (rng4 = SampleState.rng_state, or NULL). */
float orc_decode_synth_q(uint64_t seq_id, uint64_t cookie, const uint64_t *rng4, uint32_t idx);

/* n descriptors through the reference's process_descriptor
 * (cu/worker.cu:25-64) and attention_decode_step_fixed128
 * (cu/attention_decode.cu:60-204): slot and seq_len rules, fp16 q from
 * q_buf[slot] or the synthesized query, the attention of
 * test/test_bench.cu:109-150 (fp32), the kernel's argmax tie order, the
 * cycle estimate.  o_rows (fp32 [n][128], may be NULL) gets each
 * descriptor's output.  A block index >= n_blocks gives token_id
 * UINT32_MAX and cycles 0.  Returns the number of such records. */
uint32_t orc_decode_steps(const Descriptor *descs, uint32_t n, const uint8_t *arena,
                          uint64_t block_size, uint64_t n_blocks, const uint64_t *rng4,
                          const uint16_t *q_buf, uint32_t io_slots, float *o_rows,
                          Completion *comps);
uint16_t orc_f32_to_f16_rne(float f);

/* reference src/hw_worker_sim.c:22-59 run over a FIFO stream; returns the
 * number of done records, writes decoded token count. */
uint32_t orc_worker_sim_stream(const hw_desc_t *in, uint32_t n, hw_desc_t *done,
                               uint64_t *decoded_tokens);

/* reference src/infer_submit.c:17-30 descriptor fill. */
void orc_submit_desc(uint32_t gpu_group_id, uint32_t kv_arena_id, uint32_t rollout_id,
                     uint64_t kv_offset, uint64_t delta_offset, uint32_t prefix_id,
                     uint32_t seq_len, uint32_t max_tokens, hw_desc_t *out);

/* reference cu/sample.cu:40-123 for one row with the uniform injected
 * (r = (u24 & 0xFFFFFF) / 2^24); uses expf.  fma_cum selects whether the
 * top-p walk accumulates with one fused multiply-add.  scratch: V floats. */
uint32_t orc_sample_row(const float *logits, uint32_t V, float temperature,
                        uint32_t top_k, float top_p, uint32_t u24, int fma_cum,
                        float *scratch);

/* Uniform for (seed, rollout_id, step): Philox4x32-10 with key = seed and
 * counter = {step lo, step hi, rollout_id, 0}; low 24 bits of word 0. */
uint32_t orc_sample_u24(uint64_t seed, uint32_t rollout_id, uint64_t step);

/* reference cu/gpu_scheduler.cu:26-83 pass loop.  All requests are in the
 * ring before pass 0 unless arrival_pass is given (request i becomes
 * visible at pass arrival_pass[i]).  max_admit: requests consumed per pass
 * (1 = reference).  drop_when_full: 1 = reference behaviour (a request that
 * finds no free slot is consumed and lost), 0 = leave it queued.
 * Stops at the sentinel (request_id == UINT64_MAX), or when every request
 * has finished, or after max_passes.  Returns the number of done records. */
uint32_t orc_scheduler_run(const RolloutRequest *reqs, uint32_t n_reqs,
                           const uint32_t *arrival_pass, uint32_t max_admit,
                           int drop_when_full, uint32_t max_passes,
                           RolloutDone *dones, uint32_t *done_pass,
                           GpuRolloutState *state, uint32_t *passes_run,
                           uint32_t *admit_pass, uint32_t max_slots);

/* Philox U(0,1) reward of the rollout loop's RT_REWARD_PHILOX mode. */
float orc_reward_u01(uint64_t seed, uint32_t request_lo);

/* Group-normalised advantages, group size G (n % G == 0):
 * A_i = (r_i - mean_g) / (std_g + eps), population std, every sum in fp32
 * in index order, no fused multiply-add. */
void orc_grpo_advantages(const float *rewards, uint32_t n, uint32_t G, float eps,
                         float *adv);

#ifdef __cplusplus
}
#endif
