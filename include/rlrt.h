/*
 * rlrt.h - B200 entry points of the GPU-resident rollout hot path.
 *
 * The reference launches its kernels with <<<>>> from driver files that
 * declare them by hand (reference src/main.c:39-41,
 * bench/bench_gpu_scheduler.cu:8-9).  This runtime exposes each kernel as a
 * plain C function instead, so host code stays in C: device pointers and
 * sizes in, an int status out (RT_OK or a negative RT_E* code; details via
 * rt_last_error()).  `stream` is a cudaStream_t passed as void* (NULL = the
 * legacy default stream).  Nothing here allocates device memory unless its
 * name says create/alloc.
 */
#pragma once
#include <stddef.h>
#include <stdint.h>
#include "request.h"
#include "ring.h"
#include "kv_prefix.h"

#ifdef __cplusplus
extern "C" {
#endif

#define RT_OK            0
#define RT_EINVAL       (-1)   /* bad argument or shape */
#define RT_ECUDA        (-2)   /* CUDA runtime/driver error */
#define RT_ETIMEOUT     (-3)   /* a bounded device wait expired */
#define RT_ENOMEM       (-4)   /* workspace/allocation too small */
#define RT_EDEVICE      (-5)   /* kernel reported a bad index (see message) */

/* Message of the last failing call on this thread ("" if none). */
const char *rt_last_error(void);

/* Library build tag, e.g. "rlrt-b200 sm_100a". */
const char *rt_version(void);

/* ------------------------------------------------------------------------
 * Paged GQA decode attention (no reference counterpart: the reference's
 * attention_decode_step_fixed128, cu/attention_decode.cu:60-204, covers one
 * head and one 32-token block; this generalises it to paged GQA).
 *
 *   q        bf16 [num_seqs][num_q_heads][128]
 *   kv_arena bf16 pages, layout of kv_layout.h (rt_page_elem_offset)
 *   page_table int32 [num_seqs][max_pages_per_seq]
 *   seq_lens int32 [num_seqs]   (0 <= len <= max_seq_len)
 *   out      fp32 [num_seqs][num_q_heads][128]
 *   out[b][h] = softmax(q[b][h] . K[b][h/G]^T * scale) . V[b][h/G]
 * with G = num_q_heads / num_kv_heads in {1, 2, 4, 8}.
 * ---------------------------------------------------------------------- */
typedef struct {
    uint32_t num_seqs;
    uint32_t num_q_heads;
    uint32_t num_kv_heads;
    uint32_t head_dim;           /* must be 128 */
    uint32_t max_pages_per_seq;  /* page-table row stride */
    uint32_t max_seq_len;        /* upper bound on every seq_lens[b] */
    uint64_t arena_pages;        /* pages addressable in kv_arena */
    float    scale;              /* softmax scale, usually 1/sqrt(128) */
    uint32_t chunk_pages;        /* pages per split-K work unit; 0 = auto */
} rt_attn_params_t;

/* Device scratch the attention call needs (split-K partials, per-(seq,head)
 * arrival counters, one error word).  Zero it once (rt_attn_workspace_init)
 * before the first call; every call leaves the counters at zero again.
 * Calls sharing one workspace must not overlap on the GPU. */
size_t rt_attn_workspace_bytes(const rt_attn_params_t *p);
int rt_attn_workspace_init(void *workspace, size_t bytes, void *stream);

int rt_paged_decode_attention(const rt_attn_params_t *p,
                              const void *q, const void *kv_arena,
                              const int32_t *page_table, const int32_t *seq_lens,
                              float *out, void *workspace, size_t workspace_bytes,
                              void *stream);

/* Read back (and clear) the device error word of a workspace.  0 = no
 * error; otherwise RT_EDEVICE-class codes: 1 = seq_len above
 * max_seq_len / page capacity, 2 = page index outside the arena,
 * 3 = pipeline wait timed out.  Synchronises the stream. */
int rt_attn_workspace_error(void *workspace, void *stream, int32_t *code);

/* Grid/tile parameters the launcher picked for these params (for tests and
 * reports): chunk_pages actually used and the number of CTAs launched. */
int rt_attn_plan(const rt_attn_params_t *p, uint32_t *chunk_pages,
                 uint32_t *max_chunks, uint64_t *ctas);

/* ------------------------------------------------------------------------
 * Fused sampler (replaces reference cu/sample.cu:40-123 sample_token).
 *
 * One call samples one token per row of fp32 logits with the reference's
 * selection semantics, exactly:
 *   1. temperature > 0: logits *= 1.0f / temperature (fp32);
 *   2. 0 < top_k < vocab: keep entries >= the min(top_k,256)-th largest
 *      value counted with multiplicity among values > -FLT_MAX (ties at the
 *      cutoff survive); the rest become -FLT_MAX;
 *   3. 0 < top_p < 1: m = max, sum = sequential fp32 sum of __expf(l - m) in
 *      index order, inv = 1.0f / sum, walk cum += __expf(l - m) * inv and
 *      return the first index with cum >= r (top_p only selects this walk;
 *      there is no nucleus truncation, as in the reference); otherwise
 *      walk cum += __expf(l - m) / sum; vocab - 1 if the walk never reaches r.
 * The uniform r = (u & 0xFFFFFF) / 2^24 comes from Philox4x32-10 with
 * key = seed and counter = {step lo, step hi, rollout_id, 0}, u = word 0
 * (the reference draws it from per-trajectory xoshiro256** state instead).
 * Logits are read once and not modified (the reference filters in place).
 * ---------------------------------------------------------------------- */
typedef struct {
    float    temperature;
    uint32_t top_k;          /* reference SampleState.top_k is uint16 */
    float    top_p;
    uint32_t rollout_id;     /* Philox counter word 2 */
    uint64_t step;           /* Philox counter words 0..1 */
} rt_sample_row_t;

typedef struct {
    uint32_t num_rows;
    uint32_t vocab;          /* 1 .. 32768 */
    uint64_t row_stride;     /* floats between consecutive rows (>= vocab) */
    uint64_t seed;           /* Philox key */
    uint32_t fused_cum;      /* 1: top-p walk accumulates with one fma
                                (matches nvcc's default contraction of the
                                reference), 0: separate multiply and add */
} rt_sample_params_t;

/* logits fp32 [num_rows][row_stride] (device), rows [num_rows] (device),
 * tokens_out uint32 [num_rows] (device). */
int rt_sample_rows(const rt_sample_params_t *p, const float *logits,
                   const rt_sample_row_t *rows, uint32_t *tokens_out, void *stream);

/* The 24-bit uniform rt_sample_rows uses for (seed, rollout_id, step). */
uint32_t rt_sample_uniform24(uint64_t seed, uint32_t rollout_id, uint64_t step);

/* ------------------------------------------------------------------------
 * Synthetic data (seeded, counter-based, reproducible on any GPU).
 * ---------------------------------------------------------------------- */
/* n bf16 values ~ N(mean, std) from Philox4x32-10(key = seed,
 * counter = {i/4, stream, 0, 0}). */
int rt_fill_normal_bf16(void *dst, uint64_t n, uint64_t seed, uint32_t stream,
                        float mean, float std, void *s);
/* n fp32 values ~ N(mean, std), same stream definition. */
int rt_fill_normal_f32(float *dst, uint64_t n, uint64_t seed, uint32_t stream,
                       float mean, float std, void *s);

#ifdef __cplusplus
}
#endif
