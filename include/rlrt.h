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
#include "arena.h"
#include "reward.h"
#include "attention_decode.h"

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
    uint32_t kv_evict_first;     /* 1: KV loads carry an L2 evict-first hint
                                    (pure streaming); 0: normal caching, so
                                    pages shared by several sequences (a
                                    copy-on-write prefix) are reused from L2 */
} rt_attn_params_t;

/* Device scratch the attention call needs (split-K partials, per-(seq,head)
 * arrival counters, the work dispenser, one error word).  Zero it once
 * (rt_attn_workspace_init) before the first call; every call leaves the
 * counters and the dispenser at zero again.
 * Calls sharing one workspace must not overlap on the GPU. */
size_t rt_attn_workspace_bytes(const rt_attn_params_t *p);
int rt_attn_workspace_init(void *workspace, size_t bytes, void *stream);

int rt_paged_decode_attention(const rt_attn_params_t *p,
                              const void *q, const void *kv_arena,
                              const int32_t *page_table, const int32_t *seq_lens,
                              float *out, void *workspace, size_t workspace_bytes,
                              void *stream);

/* Same computation as rt_paged_decode_attention, for callers that cannot
 * allocate device memory where they run it: code under a no-allocation
 * hot-path rule (the reference's HotpathGuard treats any allocation after
 * activation as a violation), hosts whose device memory belongs to an
 * allocator that must not be bypassed, and loops where cudaMalloc/cudaFree
 * would synchronise the device.  No counterpart in the reference.
 *
 * The split-K scratch is a 32 MiB array in the library's own device memory
 * (every GPU that loads the library holds it until exit); shapes needing
 * more (rt_attn_workspace_bytes > 32 MiB) are rejected with RT_ENOMEM.  It
 * calls no allocator.  The first call on a device (and the first after a
 * cudaDeviceReset there) looks up the array's address with that device
 * current; make that first call before any stream capture.  All calls share
 * the one array and each call clears its error word and counters, so calls
 * that overlap on the GPU (any streams) race and must be serialised by the
 * caller.  Index errors (a page id outside the arena, a length above
 * max_seq_len) are caught on the device, the access is clamped, and the
 * code is kept in the array until the next call: read it with
 * rt_paged_decode_attention_noalloc_error before calling again. */
int rt_paged_decode_attention_noalloc(const rt_attn_params_t *p,
                                      const void *q, const void *kv_arena,
                                      const int32_t *page_table, const int32_t *seq_lens,
                                      float *out, void *stream);

/* Error word of the last rt_paged_decode_attention_noalloc call on the
 * current device, with the codes of rt_attn_workspace_error; reads and
 * clears it (and any part-counted arrival counters) in the built-in array.
 * Allocates nothing; synchronises the stream.  No counterpart in the
 * reference. */
int rt_paged_decode_attention_noalloc_error(int32_t *code, void *stream);

/* Shared-prefix ("cascade") decode attention.  In a GRPO group every
 * rollout starts from the same prompt, so its sequences' page tables begin
 * with the same pages (the copy-on-write prefix of kv_prefix.h).  A group
 * record lists such sequences; their common full pages are read from HBM once
 * per group and each page is multiplied against every member's queries in
 * one tensor-core tile (16 query rows = 16/G sequences x G heads), instead of
 * once per sequence.  The sequences' remaining pages are processed as in
 * rt_paged_decode_attention and the two parts merged exactly (log-sum-exp),
 * so the result equals rt_paged_decode_attention's to fp32 rounding.
 *
 * Contract (device-side violations set error 4 and are otherwise skipped):
 *  - members[i] < num_seqs, 1 <= n_members <= 16, a sequence in at most one
 *    live group;
 *  - page_table[m][0 .. shared_pages) is the same for every member m (the
 *    pages are taken from members[0]'s row) and shared_pages * 16 <=
 *    seq_lens[m];
 *  - skip_pages[m] == shared_pages for every member, 0 for a sequence in no
 *    group, and shared_pages <= gp->max_shared_pages.
 * groups[0 .. *n_groups) are live; n_groups and skip_pages are read on the
 * device, so a CUDA graph can rebuild them every step. */
typedef struct {
    uint32_t n_members;
    uint32_t shared_pages;       /* full 16-token pages common to all members */
    uint32_t members[16];        /* sequence indices */
} rt_attn_group_t;

typedef struct {
    uint32_t max_groups;         /* capacity of the groups array */
    uint32_t max_shared_pages;   /* bound on every shared_pages */
    uint32_t chunk_pages;        /* shared pages per work item; 0 = auto (16, or 32
                                    when max_shared_pages > 64) */
    uint32_t reserved;
} rt_attn_group_params_t;

size_t rt_attn_grouped_workspace_bytes(const rt_attn_params_t *p,
                                       const rt_attn_group_params_t *gp);

int rt_paged_decode_attention_grouped(const rt_attn_params_t *p,
                                      const rt_attn_group_params_t *gp,
                                      const void *q, const void *kv_arena,
                                      const int32_t *page_table, const int32_t *seq_lens,
                                      const rt_attn_group_t *groups, const uint32_t *n_groups,
                                      const uint32_t *skip_pages,
                                      float *out, void *workspace, size_t workspace_bytes,
                                      void *stream);

/* Read back (and clear) the device error word of a workspace.  0 = no
 * error; otherwise RT_EDEVICE-class codes: 1 = seq_len above
 * max_seq_len / page capacity, 2 = page index outside the arena,
 * 3 = pipeline wait timed out, 4 = group record breaks the contract of
 * rt_paged_decode_attention_grouped.  After a non-zero code the split-K
 * arrival counters of the last call may be left part-counted; this call
 * clears them too, so the workspace is ready for the next call.
 * Synchronises the stream. */
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
    uint64_t seed;           /* Philox key */
} rt_sample_row_t;

typedef struct {
    uint32_t num_rows;
    uint32_t vocab;          /* 1 .. 32768 */
    uint64_t row_stride;     /* floats between consecutive rows (>= vocab) */
    uint32_t fused_cum;      /* 1: top-p walk accumulates with one fma
                                (matches nvcc's default contraction of the
                                reference; verified bit-exact on B200),
                                0: separate multiply and add */
    const uint32_t *row_enable; /* device [num_rows] or NULL; rows whose flag
                                   is 0 are skipped and their token is left
                                   untouched */
} rt_sample_params_t;

/* logits fp32 [num_rows][row_stride] (device), rows [num_rows] (device),
 * tokens_out uint32 [num_rows] (device). */
int rt_sample_rows(const rt_sample_params_t *p, const float *logits,
                   const rt_sample_row_t *rows, uint32_t *tokens_out, void *stream);

/* The 24-bit uniform rt_sample_rows uses for (seed, rollout_id, step). */
uint32_t rt_sample_uniform24(uint64_t seed, uint32_t rollout_id, uint64_t step);

/* Producer chunk maxima.  chunk_max fp32 [num_rows][cmax_stride] (device)
 * holds, for chunk c of a row, the maximum of logits[16c .. 16c+15] (the
 * last chunk is partial), or NaN when one of them is NaN.  The kernel that
 * writes the logits can write them at little cost (the rollout loop's
 * logits kernel does); rt_logits_chunk_max computes them from the logits.
 * cmax_stride >= rt_chunk_max_stride(vocab), a multiple of 4. */
uint32_t rt_chunk_max_stride(uint32_t vocab);
int rt_logits_chunk_max(const float *logits, uint32_t num_rows, uint32_t vocab,
                        uint64_t row_stride, float *chunk_max, uint32_t cmax_stride,
                        void *stream);

/* rt_sample_rows given the logits' chunk maxima (16-byte aligned): the same
 * tokens, bit for bit, for any logits; the common row reads its chunk
 * maxima and only the chunks that can hold a top-k survivor, not the whole
 * row.  Chunk maxima that do not match the logits give undefined tokens. */
int rt_sample_rows_cmax(const rt_sample_params_t *p, const float *logits,
                        const float *chunk_max, uint32_t cmax_stride,
                        const rt_sample_row_t *rows, uint32_t *tokens_out, void *stream);

/* ------------------------------------------------------------------------
 * GPU-resident rollout loop.
 *
 * Replaces reference cu/gpu_scheduler.cu:26-83 (rollout_worker, whose
 * per-pass "decode" is a token counter).  Each pass, on the GPU and without
 * host involvement:
 *   1. commit the tokens sampled in the previous pass
 *      (tokens_generated++ per decoding slot);
 *   2. admit up to max_admit requests, in ring order, each into the lowest
 *      free slot, initialising the reference's GpuRolloutSlot fields
 *      exactly as cu/gpu_scheduler.cu:40-55 (request_id low 32 bits,
 *      rng_state {s, s^0x9e37.., (s<<17)^0x3c6e.., ~s}); request_id ==
 *      UINT64_MAX stops the loop at once; with drop_when_full a request that
 *      finds no free slot is consumed and lost (reference), otherwise it
 *      stays queued (backpressure);
 *   3. in slot order, finish every active slot whose tokens_generated has
 *      reached max_tokens: push RolloutDone{request_id low 32, slot,
 *      tokens, reward, 0} (reward (tokens & 0xFF)/255 in RT_REWARD_MOCK),
 *      free the slot, bump *step_count;
 *   4. decode one token for every remaining active slot:
 *      RT_ROLLOUT_DECODE_FULL: synthesize q and the new token's K/V
 *      (Philox N(0,1)), copy-on-write the partial last page of a shared
 *      prefix on the first write, paged GQA attention over the slot's
 *      context, synthetic logits ~ N(0, logit_std) (Philox key = request
 *      rng_seed, counter = (token index, request low 32)), fused sampling
 *      with the slot's temperature/top_k/top_p;
 *      RT_ROLLOUT_DECODE_NONE: no math (the reference's counter).
 * An array source may carry per-request arrival times (rt_rollout_io_t
 * arrivals): a request is admitted no earlier than its arrival, which
 * replays an open-loop arrival process (e.g. Poisson) on the device.
 * A request routes to a shared prefix through request_id bits 32..63
 * (prefix id + 1, see request.h); the prefix's pages are registered with
 * rt_rollout_set_prefix.  Token ids land in `trajectories` row r =
 * the request's consume index (0, 1, 2, ... in ring/array order).
 * ---------------------------------------------------------------------- */
#define RT_ROLLOUT_DECODE_NONE  0u
#define RT_ROLLOUT_DECODE_FULL  1u
#define RT_ROLLOUT_DECODE_MODEL 2u   /* as FULL, with q/K/V and logits from model weights
                                        (rt_rollout_set_model) instead of Philox */
#define RT_REWARD_MOCK          0u   /* (tokens & 0xFF) / 255 (reference) */
#define RT_REWARD_PHILOX        1u   /* U(0,1): Philox(key = reward_seed, ctr = {request low 32}) */
#define RT_PREFIX_ATTN_GROUPED       0u  /* default: rt_paged_decode_attention_grouped over
                                           groups of slots with the same prefix */
#define RT_PREFIX_ATTN_PER_SEQUENCE  1u  /* rt_paged_decode_attention, every slot on its own */
#define RT_ARRIVAL_PASS  0u  /* arrivals[i] is a pass index (0 = the first pass): deterministic */
#define RT_ARRIVAL_NS    1u  /* arrivals[i] is ns of GPU global time since the first pass began */

typedef struct {
    uint32_t num_q_heads;       /* 32 */
    uint32_t num_kv_heads;      /* 8 (page bytes = num_kv_heads * 8 KiB) */
    uint32_t vocab;             /* <= 32768 */
    uint32_t max_slots;         /* concurrent rollouts, <= GPU_MAX_ROLLOUTS */
    uint32_t max_context;       /* tokens per rollout incl. prefix */
    uint32_t max_new_tokens;    /* per rollout (trajectory row length) */
    uint32_t max_admit;         /* requests admitted per pass (1 = reference) */
    uint32_t drop_when_full;    /* 1 = reference, 0 = backpressure */
    uint32_t decode_mode;       /* RT_ROLLOUT_DECODE_* */
    uint32_t reward_mode;       /* RT_REWARD_* */
    uint64_t reward_seed;
    float    logit_std;         /* synthetic logits ~ N(0, logit_std) */
    uint32_t max_prefixes;      /* prefix ids 0 .. max_prefixes-1 */
    uint32_t max_prefix_pages;  /* total pages over all registered prefixes */
    uint64_t max_passes;        /* stop with RT_ETIMEOUT after this many passes */
    uint32_t idle_timeout_ms;   /* ring source: stop with RT_ETIMEOUT when idle this long */
    uint32_t chunk_pages;       /* attention split-K chunk (0 = auto: 16 pages when
                                   max_context exceeds 64 pages, else the attention
                                   plan's rule) */
    uint32_t prefix_attention;  /* RT_PREFIX_ATTN_*: how slots sharing a prefix attend */
} rt_rollout_config_t;

typedef struct {
    RequestRing *ring;                 /* request source: a ring ... */
    const RolloutRequest *requests;    /* ... or a device array (ring == NULL) */
    uint32_t n_requests;
    DoneRing *done_ring;               /* done sink: a ring ... */
    RolloutDone *dones;                /* ... or a device array (capacity n_rows) */
    GpuRolloutState *state;            /* device, reference layout; zeroed at launch */
    uint64_t *step_count;              /* device, may be NULL */
    uint32_t *trajectories;            /* device [n_rows][max_new_tokens], may be NULL */
    float *rewards;                    /* device [n_rows], may be NULL */
    uint32_t n_rows;
    uint32_t arrival_unit;             /* RT_ARRIVAL_* of `arrivals` */
    const uint64_t *arrivals;          /* array source only: device [n_requests] or NULL.
                                          Request i may be admitted only in a pass that
                                          starts at or after arrivals[i]; requests are
                                          taken in order, so a request that has not
                                          arrived holds back the ones behind it. */
} rt_rollout_io_t;

typedef struct {
    uint64_t passes;
    uint64_t tokens;          /* tokens generated (committed) */
    uint32_t consumed;        /* requests taken from the source (incl. dropped) */
    uint32_t admitted;
    uint32_t dropped;
    uint32_t done;
    uint32_t max_active;
    uint32_t stopped_by_sentinel;
    int32_t  error;           /* 0, or RT_ETIMEOUT / RT_EDEVICE */
    int32_t  attn_error;      /* attention workspace error word */
    int32_t  model_error;     /* model decode: projection kernel error word */
    uint32_t pad;
} rt_rollout_stats_t;

typedef struct rt_rollout rt_rollout_t;

/* Allocate the engine's device state and reserve its private KV pages
 * (max_slots x ceil((max_new_tokens + 16) / 16) blocks) from `arena`,
 * whose block_size must be the page size (num_kv_heads * 8 KiB). */
int rt_rollout_create(const rt_rollout_config_t *cfg, KVArena *arena, rt_rollout_t **out);
int rt_rollout_destroy(rt_rollout_t *eng);

/* Register the pages (arena block indices, host array) of shared prefix
 * `prefix_id` holding `token_len` tokens (the prefix_id of
 * kv_prefix_register).  A partial last page is copied on first write. */
int rt_rollout_set_prefix(rt_rollout_t *eng, uint32_t prefix_id, const int32_t *pages,
                          uint32_t n_pages, uint32_t token_len);

/* Launch the loop asynchronously on `stream`.  It ends at the sentinel,
 * when an array source is exhausted and no rollout is active, or on error. */
int rt_rollout_launch(rt_rollout_t *eng, const rt_rollout_io_t *io, void *stream);

/* Per-kernel device time of a host-stepped replay of the loop. */
typedef struct {
    uint64_t passes;
    uint64_t attn_launches;       /* passes with at least one active slot */
    uint64_t sample_rows;         /* active slot-passes (rows sampled) */
    double ms_schedule, ms_prepare, ms_attention, ms_logits, ms_sample;
    double attn_bytes_logical;    /* sum over slots of context x K/V bytes per token */
    double attn_bytes_unique;     /* same with each shared prefix counted once per pass */
} rt_rollout_profile_t;

/* Run the loop pass by pass from the host, with CUDA events around each
 * kernel (same kernels and data as rt_rollout_launch); synchronous. */
int rt_rollout_profile(rt_rollout_t *eng, const rt_rollout_io_t *io, void *stream,
                       rt_rollout_profile_t *out);

/* rt_rollout_profile with a callback after every pass (the stream is
 * synchronised, the engine's buffers hold that pass's inputs and outputs);
 * a nonzero return stops the replay there.  For inspection and tests. */
typedef int (*rt_rollout_pass_hook_t)(void *user, uint64_t pass);
int rt_rollout_profile_hook(rt_rollout_t *eng, const rt_rollout_io_t *io, void *stream,
                            rt_rollout_profile_t *out, rt_rollout_pass_hook_t hook, void *user);

/* Device buffers of a full-decode engine (read them between passes). */
typedef struct {
    const void *q;                   /* bf16 [max_slots][num_q_heads][128] */
    const float *attn_out;           /* fp32 [max_slots][num_q_heads][128] */
    const int32_t *page_table;       /* [max_slots][max_pages] */
    const int32_t *seq_lens;         /* [max_slots] (0 = idle this pass) */
    const rt_attn_group_t *groups;   /* [max_groups]; NULL when not grouped */
    const uint32_t *n_groups;        /* [1] */
    const uint32_t *skip_pages;      /* [max_slots] */
    uint32_t max_pages;
    uint32_t max_groups;
    const float *logits;             /* fp32 [max_slots][vocab] */
    const uint32_t *tokens;          /* [max_slots] sampled this pass */
    const uint32_t *enable;          /* [max_slots] 1 = decoded this pass */
    const rt_sample_row_t *sample_rows; /* [max_slots] sampling parameters of this pass */
    const void *hidden_in;           /* model decode: bf16 [max_slots][d_model] embeddings */
    const float *qkv;                /* model decode: fp32 [max_slots][(q + 2 kv heads) * 128] */
    const void *hidden_out;          /* model decode: bf16 [max_slots][d_model] = attn_out */
    const uint32_t *embed_tokens;    /* model decode: [max_slots] token embedded this pass */
} rt_rollout_buffers_t;
int rt_rollout_buffers(rt_rollout_t *eng, rt_rollout_buffers_t *out);

/* Model weights of a RT_ROLLOUT_DECODE_MODEL engine (device bf16, rows of
 * d_model = num_q_heads * 128 elements, K contiguous; the engine keeps the
 * pointers).  Each pass then runs, for every decoding slot s:
 *   x_s      = embed[last token of s]            (token 0 before the first)
 *   [q|k|v]  = x_s . w_qkv^T                     (cuBLAS GEMM, fp32)
 *   q, and k / v written into the slot's page at its position (bf16)
 *   o_s      = paged GQA attention (as FULL)
 *   logits_s = bf16(o_s) . w_lm^T                (tensor-core GEMM, fp32)
 *   token    = fused sampling of logits_s (as FULL).
 * embed [vocab][d_model]; w_qkv [(num_q_heads + 2 num_kv_heads) * 128]
 * [d_model] (q rows, then k rows per kv head, then v rows per kv head);
 * w_lm [vocab][d_model].  Must be called before the first launch.  The
 * first call also creates the engine's cuBLAS handle and its 32 MiB
 * workspace (the QKV product). */
typedef struct {
    const void *embed;
    const void *w_qkv;
    const void *w_lm;
    uint32_t d_model;
    uint32_t reserved;
} rt_model_weights_t;
int rt_rollout_set_model(rt_rollout_t *eng, const rt_model_weights_t *w);

/* Model prefill of a registered prefix (RT_ROLLOUT_DECODE_MODEL engine with
 * its weights attached): `tokens` (device, uint32 [n_tokens]) are the
 * prompt's token ids and n_tokens the token length the prefix was
 * registered with; for every position i the K and V rows
 *   [k | v] = bf16(embed[tokens[i]] . w_qkv[k and v rows]^T)
 * are written into the prefix's page holding i (a tensor-core GEMM over
 * 4,096 positions at a time).  A token id >= vocab is replaced by 0 and
 * flags RT_EDEVICE in the model error word.  Stream-ordered; it shares
 * scratch with the engine's launches, so it must not overlap one. */
int rt_rollout_prefill(rt_rollout_t *eng, uint32_t prefix_id, const uint32_t *tokens,
                       uint32_t n_tokens, void *stream);

/* Wait for the loop (stream sync) and read its counters. */
int rt_rollout_wait(rt_rollout_t *eng, void *stream, rt_rollout_stats_t *stats);

/* Synthetic logits of the loop for (seed, request low 32, token index):
 * out[v] = logit_std * N(0,1), v < vocab (device); used to replay a run. */
int rt_logits_synth(float *out, uint32_t vocab, uint64_t seed, uint32_t request_lo,
                    uint64_t token_index, float logit_std, void *stream);

/* Host side of a ring-fed run, in C (the producer/consumer loop of the
 * reference's bench driver, bench/bench_gpu_scheduler.cu:57-83): push the
 * n requests into `rq` as space allows (then the stop sentinel when
 * send_sentinel), while draining `dn` into `dones` until n_expected records
 * arrived.  Returns the number drained, or -1 when timeout_ms passed first
 * (the records drained so far are in `dones`). */
int64_t rt_host_pump(RequestRing *rq, const RolloutRequest *reqs, uint32_t n, DoneRing *dn,
                     RolloutDone *dones, uint32_t n_expected, int send_sentinel,
                     uint32_t timeout_ms);

/* rt_host_pump with open-loop pacing: request i is pushed no earlier than
 * arrival_ns[i] nanoseconds (CLOCK_MONOTONIC) after the call starts, in
 * order (arrival_ns non-decreasing; NULL = as fast as the ring allows).
 * When done_ns is given, done_ns[k] receives the time, on the same clock,
 * at which dones[k] was drained.  Returns as rt_host_pump. */
int64_t rt_host_pump_paced(RequestRing *rq, const RolloutRequest *reqs, const uint64_t *arrival_ns,
                           uint32_t n, DoneRing *dn, RolloutDone *dones, uint64_t *done_ns,
                           uint32_t n_expected, int send_sentinel, uint32_t timeout_ms);

/* Drop-in for the reference launch
 *     rollout_worker<<<1, 32>>>(req_ring, done_ring, state, step_count)
 * (reference bench/bench_gpu_scheduler.cu:55): a persistent single-CTA
 * kernel with the reference's pass semantics and counter-only decode,
 * returning immediately; it exits at the request_id == UINT64_MAX sentinel
 * (or after idle_timeout_ms without work, flagging RT_ETIMEOUT). */
int rt_launch_rollout_worker(RequestRing *req_ring, DoneRing *done_ring,
                             GpuRolloutState *state, uint64_t *step_count,
                             uint32_t idle_timeout_ms, void *stream);

/* Counters of the last rt_launch_rollout_worker on the current device
 * (reads device memory on `stream`; safe while the worker runs). */
int rt_rollout_worker_stats(void *stream, rt_rollout_stats_t *stats);

/* ------------------------------------------------------------------------
 * Per-step CommandRing decode path: the persistent decode worker and the
 * fixed128 attention step (reference cu/worker.cu:25-131,
 * cu/attention_decode.cu:16-204).
 *
 * The step, per Descriptor: seq_len = num_kv_blocks (0 -> 1) clamped to 32
 * tokens of the 16 KiB fp16 block arena[kv_block_offset] (K plane then V
 * plane, kv_layout.h); slot = io_slots ? output_token_offset & (io_slots-1)
 * : 0; q = q_buffer[slot] (fp16 [128]) or, when q_buffer is NULL, the
 * reference's synthesized query (seq_id, reward_cookie and, when sample_st
 * is given, sample_st->rng_state); o = softmax(q.K^T / sqrt(128)).V,
 * written to o_buffer[slot] (fp32 [128]) when given; token_id = argmax o
 * with the reference's tie order (lowest d mod 32, then lowest d / 32);
 * cycle_estimate = ceil(seq_len/16) * 128 * 24.  The fp32 evaluation order
 * is the reference kernel's, so o and token_id are identical to it.
 * ---------------------------------------------------------------------- */
typedef struct {
    uint64_t consumed;        /* CommandRing records taken, sentinels included (final) */
    uint64_t completed;       /* Completion records pushed (== step_count increments) */
    uint32_t published;       /* work descriptors handed to the worker warps */
    uint32_t sentinels;       /* stop sentinels taken (final) */
    uint32_t comp_ring_full;  /* times a finished completion found the CompletionRing full */
    int32_t  error;           /* RT_OK, RT_ETIMEOUT (a bounded wait expired) or
                                 RT_EDEVICE (kv_block_offset outside the arena) */
    uint32_t bad_block;       /* first out-of-range kv_block_offset */
    uint32_t workers;         /* worker warps in the grid */
    uint32_t finished;        /* 1 once the worker kernel has stopped */
    uint32_t pad;
} rt_decode_worker_stats_t;

/* Drop-in for the reference launch
 *     decode_worker<<<num_SMs, 32, 3 * 16384>>>(cmd_ring, &kv_arena, comp_ring,
 *         sample_st, q_buffer, o_buffer, io_slots, step_count)
 * (reference src/main.c:229-235, kernel cu/worker.cu:77-131).  Returns
 * after the launch.  One pump warp takes CommandRing records in batches
 * (the ring keeps one consumer) and delivers Completions in ring order
 * (the CompletionRing keeps one producer); the other warps of one CTA per
 * SM run the step.  `arena` is the host KVArena (its device base and
 * block_size, >= 16 KiB, are read here); sample_st, q_buffer, o_buffer and
 * step_count are device pointers (each may be NULL).  The worker stops at
 * the stop_sentinels-th record with seq_id == UINT64_MAX (0 = the device's
 * SM count, one per reference worker warp as src/main.c:179-190 pushes);
 * records behind it stay in the ring.  A kv_block_offset outside the
 * arena yields a Completion with token_id = UINT32_MAX, cycles_taken = 0
 * and flags RT_EDEVICE; idle_timeout_ms (0 = 10 s) without progress ends
 * the worker with RT_ETIMEOUT.  One decode worker per device at a time. */
int rt_launch_decode_worker(CommandRing *ring, const KVArena *arena, CompletionRing *comp_ring,
                            const SampleState *sample_st, const void *q_buffer, float *o_buffer,
                            uint32_t io_slots, uint64_t *step_count, uint32_t stop_sentinels,
                            uint32_t idle_timeout_ms, void *stream);

/* Counters of the last rt_launch_decode_worker on the current device
 * (reads device memory on `stream`; safe while the worker runs). */
int rt_decode_worker_stats(void *stream, rt_decode_worker_stats_t *stats);

/* The fixed128 step over n device-resident Descriptors (16-byte aligned),
 * one warp each, without rings: the reference's
 * attention_decode_step_fixed128 as called by process_descriptor
 * (cu/worker.cu:30-51), results[i] as its DecodeStepResult
 * (include/attention_decode.h).  A record whose block lies outside the
 * arena gets path_kind DECODE_PATH_STUB and token_id UINT32_MAX. */
int rt_attention_fixed128(const Descriptor *descs, uint32_t n, const KVArena *arena,
                          const SampleState *sample_st, const void *q_buffer, float *o_buffer,
                          uint32_t io_slots, DecodeStepResult *results, void *stream);

/* Host side of a CommandRing run, in C (the dispatch / poll / shutdown
 * loop of reference src/main.c:121-190): push the n descriptors as ring
 * space allows, then n_sentinels stop records, while draining the
 * CompletionRing into `out` until n_expected records arrived.  Returns
 * the number drained, or -1 when timeout_ms passed first. */
int64_t rt_host_decode_pump(CommandRing *ring, const Descriptor *descs, uint32_t n,
                            uint32_t n_sentinels, CompletionRing *comp, Completion *out,
                            uint32_t n_expected, uint32_t timeout_ms);

/* ------------------------------------------------------------------------
 * Device-side trace of the rollout loop (the GPU-side trace buffer with
 * post-hoc copyback of reference docs/tracing.md "Future").  The schedule
 * kernel appends records in the reference's 20-byte trace_entry_t layout
 * and event numbering (include/trace.h: tsc, type, rollout_id, seq), with
 * tsc the GPU's globaltimer in nanoseconds:
 *   ROLLOUT_ALLOC (request low 32, slot) and DESC_CONSUMED (request low 32,
 *   consume index) at admission; REWARD_POSTED and TRAJECTORY_DONE
 *   (request low 32, tokens generated) and ROLLOUT_FREE (request low 32,
 *   slot) at retirement; DECODE_BATCH (active slots, pass) every pass.
 * The ring lives in device memory (rt_trace_bytes(capacity), capacity a
 * power of two); when it wraps the oldest records are overwritten.
 * ---------------------------------------------------------------------- */
#define RT_TRACE_ROLLOUT_ALLOC     0u
#define RT_TRACE_ROLLOUT_FREE      1u
#define RT_TRACE_DESC_CONSUMED     4u
#define RT_TRACE_DECODE_BATCH      7u
#define RT_TRACE_REWARD_POSTED     8u
#define RT_TRACE_TRAJECTORY_DONE   10u

typedef struct __attribute__((packed)) {
    uint64_t tsc;
    uint32_t type;
    uint32_t rollout_id;
    uint32_t seq;
} rt_trace_entry_t;

size_t rt_trace_bytes(uint32_t capacity);
/* Empty the device trace ring (stream-ordered). */
int rt_trace_init(void *trace, uint32_t capacity, void *stream);
/* Attach a trace ring to an engine (NULL detaches); stream-ordered with its
 * launches, it must not be called while one is in flight. */
int rt_rollout_set_trace(rt_rollout_t *eng, void *trace);
/* Copy the ring's records back in append order: the newest min(appended,
 * capacity, max) of them into out; *appended = records appended in all. */
int rt_trace_read(const void *trace, rt_trace_entry_t *out, uint32_t max, uint64_t *appended,
                  void *stream);

/* ------------------------------------------------------------------------
 * Projections of the decode step on the tensor cores (new: the reference
 * synthesises its query with one <<<1,128>>> launch per slot and step,
 * cu/model_state.cu:6-52 and cu/query_producer.cu:5-26, and has no LM
 * head).
 *
 *   C[m][n] (+)= sum_k A[m][k] * B[n][k]
 *
 * A bf16 [M][lda] (activations, K contiguous), B bf16 [N][ldb] (a weight
 * stored [out][in], K contiguous), C fp32 [M][ldc]; fp32 accumulation.
 * K a multiple of 64; lda, ldb multiples of 8 elements; A, B 16-byte
 * aligned.  split_k > 1 divides K among CTAs: each stores its partial
 * sums into `workspace` (rt_gemm_workspace_bytes, 16-byte aligned) and a
 * second kernel adds them into C in split order, so results are
 * deterministic.  `error` is a device int32 set to 1 if a bounded wait
 * inside the kernel expired (never expected).
 * ---------------------------------------------------------------------- */
#define RT_GEMM_ACCUMULATE 1u

typedef struct {
    uint32_t M, N, K;
    uint32_t lda, ldb, ldc;  /* row strides in elements */
    uint32_t split_k;        /* 0 or 1: none */
    uint32_t flags;          /* RT_GEMM_ACCUMULATE */
} rt_gemm_params_t;

size_t rt_gemm_workspace_bytes(const rt_gemm_params_t *p);  /* 0 without K-splits */
int rt_gemm_bf16(const rt_gemm_params_t *p, const void *A, const void *B, float *C,
                 void *workspace, size_t workspace_bytes, int32_t *error, void *stream);

/* rt_gemm_bf16 that also writes C's 16-column maxima in the layout of
 * rt_logits_chunk_max (chunk_max fp32 [M][cmax_stride], cmax_stride >=
 * rt_chunk_max_stride(N)), for rt_sample_rows_cmax on an LM head's logits.
 * Without K-splits or accumulation the epilogue writes them from the
 * accumulators it already holds; otherwise they are computed from C
 * afterwards. */
int rt_gemm_bf16_chunk_max(const rt_gemm_params_t *p, const void *A, const void *B, float *C,
                           void *workspace, size_t workspace_bytes, int32_t *error,
                           float *chunk_max, uint32_t cmax_stride, void *stream);

/* ------------------------------------------------------------------------
 * Rewards and group-normalised advantages (new; the reference has only the
 * mock scorer, cu/reward.cu:4-15, never launched).
 * ---------------------------------------------------------------------- */
/* Drop-in for reward_score_kernel: descs[i].reward = scores[i] =
 * (descs[i].token_count & 0xFF) / 255 for i < n (device pointers; scores
 * may be NULL). */
int rt_reward_score(RewardDesc *descs, uint32_t n, float *scores, void *stream);

/* ------------------------------------------------------------------------
 * Device-side branch resolution over the copy-on-write prefix table
 * (replaces reference cu/kv_prefix.cu:17-23, kv_branch_resolve, and its
 * d_kv_branch_total_offset, cu/kv_prefix.cu:4-15).
 *
 * `table` is a KVPrefixTable (kv_prefix.h) in device or mapped memory, the
 * host table's bytes unchanged; branch_ids uint32 [n] and out_offsets int64
 * [n] are device pointers.  out_offsets[i] is
 *   -1                           if branch_ids[i] >= MAX_BRANCHES,
 *   branch.delta_kv_offset       if the branch's prefix id >= MAX_PREFIXES
 *                                or that prefix's refcnt is 0,
 *   prefix.kv_block_offset       otherwise.
 * These are the device kernel's semantics; the host kv_branch_total_offset
 * returns the prefix's offset whatever its refcount. */
int rt_kv_branch_resolve(const KVPrefixTable *table, const uint32_t *branch_ids,
                         int64_t *out_offsets, uint32_t n, void *stream);

/* A_i = (r_i - mean_g) / (std_g + eps) over consecutive groups of G,
 * population std; per group: fp32 sum in index order, mean = sum / G,
 * var = sum of (r - mean)^2 in index order, std = sqrt(var / G) (all
 * correctly rounded, no fused multiply-add).  n must be a multiple of G. */
int rt_grpo_advantages(const float *rewards, uint32_t n, uint32_t G, float eps, float *adv,
                       void *stream);

/* NCCL plumbing for the one cross-GPU exchange of the path: every rank
 * contributes its rollouts' rewards, every rank receives all of them in
 * rank order.  `comm` is an ncclComm_t passed as void*. */
int rt_nccl_unique_id(void *id128);
int rt_nccl_init(void **comm, int nranks, const void *id128, int rank);
int rt_nccl_destroy(void *comm);
int rt_reward_allgather(void *comm, const float *send, float *recv, uint64_t n_per_rank,
                        void *stream);
/* Wait for the stream's work with a deadline; on expiry (e.g. a peer rank
 * died) abort the communicator and return RT_ETIMEOUT instead of hanging. */
int rt_nccl_wait(void *comm, void *stream, uint32_t timeout_ms);

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
