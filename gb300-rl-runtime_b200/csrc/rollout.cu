// rollout.cu - the GPU-resident rollout loop (scheduler + decode step).
//
// Reference: cu/gpu_scheduler.cu:4-83 (rollout_worker, find_free_slot,
// release_slot).  The reference runs one persistent thread that, per pass,
// admits at most one request and then walks the 256 slots, finishing or
// "decoding" (tokens_generated++) each active one.  Here a pass is a chain of
// kernels captured once into a CUDA graph whose body repeats under a device
// controlled WHILE conditional node, so the loop runs without the host:
//
//   schedule_kernel  1 CTA x 256 threads (thread s <-> slot s): commit the
//                    previous pass's sampled tokens, admit requests, retire
//                    finished slots in slot order (RolloutDone), plan this
//                    pass (sequence lengths, sampling rows), decide whether
//                    the loop continues (cudaGraphSetConditional).
//   prepare_kernel   1 CTA per active slot: copy-on-write of a shared
//                    prefix's partial last page on the first write, q and
//                    the new token's K/V from Philox N(0,1) into the arena.
//   attention        rt_paged_decode_attention over all slots (idle slots
//                    have length 0 and cost one early-exit CTA each).
//   logits_kernel    synthetic logits ~ N(0, logit_std), Philox.
//   sampler          rt_sample_rows with the per-slot enable mask.
//
// Counter-only decode (the reference's mock) uses the same schedule pass
// with tokens_generated++ in place of the decode chain; the drop-in launcher
// rt_launch_rollout_worker runs that pass in a persistent single-CTA kernel.
#include <algorithm>
#include <cstddef>
#include <cublas_v2.h>
#include <cstdint>
#include <cstring>
#include <mutex>
#include <new>

#include "kv_layout.h"
#include "reward.h"
#include "rlrt.h"
#include "rt_common.cuh"
#include "rt_internal.h"

namespace {

constexpr int kSched = 256;  // schedule CTA: one thread per slot (GPU_MAX_ROLLOUTS)
constexpr uint64_t kDonePushLimitNs = 10000000000ull;  // 10 s bounded wait on a full done ring
#ifndef RT_PASSES_PER_ITERATION
#define RT_PASSES_PER_ITERATION 16
#endif
constexpr int kPassesPerIteration = RT_PASSES_PER_ITERATION;  // passes captured in one graph-loop body

struct RtIo {
    RequestRing *ring;
    const RolloutRequest *reqs;
    uint32_t n_reqs;
    DoneRing *done_ring;
    RolloutDone *dones;
    GpuRolloutState *state;
    unsigned long long *step_count;
    uint32_t *traj;
    float *rewards;
    uint32_t n_rows;
    uint32_t arrival_unit;      // RT_ARRIVAL_* of `arrivals`
    const uint64_t *arrivals;   // array source: per-request arrival gate, or NULL
};
static_assert(sizeof(RtIo) % 8 == 0 && sizeof(RtIo) / 8 <= 32, "RtIo is copied by one warp");

struct RtCtl {
    unsigned long long passes, tokens, idle_since;
    unsigned long long t0;  // globaltimer at the first pass (arrival clock origin)
    uint32_t consumed, admitted, dropped, done, max_active, sentinel;
    int32_t error;
    uint32_t stop;
    uint32_t groups_ok;   // the group table matches the active slot set
    uint32_t groups_act;  // active slots when it was built
};
static_assert(sizeof(RtCtl) % 8 == 0, "RtCtl is copied as 64-bit words");

struct SlotExt {
    uint32_t row, request_lo, pos, ctx_len, last_token, decoding, cow_rows;
    int32_t cow_src;
    uint64_t seed;
    uint32_t prefix;  // shared-prefix id + 1, 0 = none
    uint32_t shared;  // full prefix pages at the head of the page table (shared, read-only)
    uint32_t skip;    // of those, the pages its attention group covers (0 outside a group)
    uint32_t pad_;
};

// Device trace ring (rt_trace_*): append counter, capacity (power of two),
// records in the reference's trace_entry_t layout.
struct TraceRing {
    unsigned long long head;
    uint32_t capacity;
    uint32_t reserved;
    rt_trace_entry_t entries[1];  // capacity records
};
static_assert(offsetof(TraceRing, entries) == 16, "trace records start at 16 bytes");

__device__ __forceinline__ void trace_push(TraceRing *t, uint32_t type, uint32_t rid, uint32_t seq)
{
    if (!t)
        return;
    const unsigned long long i = atomicAdd(&t->head, 1ull);
    uint32_t *w = reinterpret_cast<uint32_t *>(&t->entries[i & (t->capacity - 1u)]);
    const uint64_t ts = rt::globaltimer_ns();
    w[0] = (uint32_t)ts;
    w[1] = (uint32_t)(ts >> 32);
    w[2] = type;
    w[3] = rid;
    w[4] = seq;
}

struct Dev {
    // configuration
    uint32_t max_slots, max_admit, drop, decode, reward_mode, vocab, maxp, ppriv, max_new;
    uint32_t hq, hkv, max_prefixes;
    uint64_t reward_seed, max_passes, idle_ns;
    float logit_std;
    // device state
    RtIo *io;
    RtCtl *ctl;
    SlotExt *ext;
    int32_t *page_table;  // [max_slots][maxp]
    int32_t *priv;        // [max_slots][ppriv]
    int32_t *seq_lens;    // [max_slots]
    uint32_t *enable;     // [max_slots]
    rt_sample_row_t *srows;
    uint32_t *tokens;     // [max_slots]
    __nv_bfloat16 *q;     // [max_slots][hq][128]
    float *attn_out;      // [max_slots][hq][128]
    __nv_bfloat16 *arena;
    float *logits;        // [max_slots][vocab]
    float *cmax;          // [max_slots][cstride] 16-column maxima of the synthetic logits
    uint32_t cstride;
    // attention items, written by the schedule kernel: [0] this pass's
    // largest per-slot chunk count, [1] the full chunks of all slots, [2 + s]
    // the full chunks of the slots before s; and the plan values they come from
    uint32_t *attn_chunks;
    uint32_t attn_cp, attn_gcp, attn_mg;
    uint32_t *pf_len, *pf_np, *pf_off;
    int32_t *pf_pages;
    // shared-prefix attention groups, rebuilt by every schedule pass
    rt_attn_group_t *groups;  // [max_groups]
    uint32_t *n_groups;       // [1]
    uint32_t *skip;           // [max_slots]
    uint32_t max_groups;      // 0 = per-sequence attention only
    // model decode (RT_ROLLOUT_DECODE_MODEL)
    const __nv_bfloat16 *w_embed, *w_qkv, *w_lm;
    __nv_bfloat16 *hin, *hout;  // [max_slots][dm]: embeddings in, attention out as bf16
    float *qkv;                 // [max_slots][qkv_n]
    uint32_t *emb_tok;          // [max_slots] token embedded this pass
    int32_t *gemm_err;          // projection kernels' error word
    uint32_t dm, qkv_n;
    float *gemm_ws;             // K-split partials of the projections
    uint64_t gemm_ws_bytes;
    uint32_t split_lm;
    TraceRing *trace;           // device trace ring, or NULL
};

__device__ __forceinline__ float reward_for(const Dev &d, uint32_t request_lo, uint32_t tokens)
{
    if (d.reward_mode == RT_REWARD_PHILOX) {
        uint32_t x[4];
        rt::philox4x32_10(request_lo, 0u, 0x52455744u, 0u, (uint32_t)d.reward_seed,
                          (uint32_t)(d.reward_seed >> 32), x);
        return (float)(x[0] >> 8) * (1.0f / 16777216.0f);
    }
    return reward_score_mock_inline(tokens);
}

// ---- request source / done sink (thread 0 only; admission reads ahead) ----
__device__ bool src_empty(const RtIo &io, const RtCtl *ctl)
{
    if (io.ring)
        return rt_load_relaxed_u32(&io.ring->cons.head) == rt_load_acquire_u32(&io.ring->prod.tail);
    return ctl->consumed + ctl->sentinel >= io.n_reqs;
}

// Reference done_ring_push semantics per attempt (overflow++ on a full
// ring); the spin is bounded so an absent consumer cannot hang the GPU.
__device__ bool sink_push(const RtIo &io, RtCtl *ctl, const RolloutDone &rec)
{
    if (!io.done_ring) {
        if (io.dones && ctl->done < io.n_rows)
            io.dones[ctl->done] = rec;
        return true;
    }
    if (done_ring_push(io.done_ring, &rec) == 0)
        return true;
    const uint64_t t0 = rt::globaltimer_ns();
    while (done_ring_push(io.done_ring, &rec) != 0) {
        __nanosleep(200);
        if (rt::globaltimer_ns() - t0 > kDonePushLimitNs)
            return false;
    }
    return true;
}

constexpr uint32_t kKeyTable = 1024;  // prefix ids grouped through a table (else a slot scan)
constexpr uint32_t kPrefillChunk = 4096;  // prompt tokens per prefill projection

__device__ __forceinline__ uint32_t ld_sys_u32(const void *p)
{
    uint32_t v;
    asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ uint16_t ld_sys_u16(const void *p)
{
    uint16_t v;
    asm volatile("ld.relaxed.sys.global.u16 %0, [%1];" : "=h"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void st_sys_u64(void *p, uint64_t v)
{
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// One 34-byte ring record (2-byte aligned) from host memory into shared
// memory: nine independent loads in flight together, not 34 serial ones.
__device__ __forceinline__ void load_request(const RolloutRequest *src, RolloutRequest *dst)
{
    const uint8_t *a = reinterpret_cast<const uint8_t *>(src);
    uint16_t *o = reinterpret_cast<uint16_t *>(dst);
    const uint32_t lead = (reinterpret_cast<uintptr_t>(a) & 3u) ? 1u : 0u;  // u16 before the words
    uint32_t w[8];
    uint16_t edge;
    if (lead) {
        edge = ld_sys_u16(a);
#pragma unroll
        for (int i = 0; i < 8; i++)
            w[i] = ld_sys_u32(a + 2 + 4 * i);
    } else {
#pragma unroll
        for (int i = 0; i < 8; i++)
            w[i] = ld_sys_u32(a + 4 * i);
        edge = ld_sys_u16(a + 32);
    }
    uint32_t k = 0;
    if (lead)
        o[k++] = edge;
#pragma unroll
    for (int i = 0; i < 8; i++) {
        o[k++] = (uint16_t)(w[i] & 0xFFFFu);
        o[k++] = (uint16_t)(w[i] >> 16);
    }
    if (!lead)
        o[k] = edge;
}

__device__ __forceinline__ uint32_t free_slot_count(const uint64_t *bitmap, uint32_t max_slots)
{
    uint32_t n = 0;
    for (uint32_t w = 0; w < (GPU_MAX_ROLLOUTS + 63) / 64; w++) {
        const uint32_t lo = w * 64u;
        if (lo >= max_slots)
            break;
        uint64_t free_bits = ~bitmap[w];
        if (max_slots - lo < 64u)
            free_bits &= (1ull << (max_slots - lo)) - 1ull;
        n += (uint32_t)__popcll(free_bits);
    }
    return n;
}


// Shared-memory copy of the loop state one schedule pass works on: loaded
// in two parallel round trips at the start of a pass, stored back at its
// end, so that the pass's serial steps (admission, retirement, loop
// control) touch no global memory except the request source and done sink.
struct SchedShared {
    GpuRolloutSlot slot[kSched];  // reference state table (slots < max_slots)
    SlotExt ext[kSched];
    uint64_t bitmap[(GPU_MAX_ROLLOUTS + 63) / 64];
    RtCtl ctl;
    RtIo io;
    union {
        // admission: requests read ahead from a RequestRing in one round trip
        RolloutRequest rq_buf[kSched];
        // after admission: the admitted slots' page-table fill, flattened
        struct {
            uint32_t f_pre[kSched + 1];  // exclusive prefix sum of entries per admission
            uint32_t f_npf[kSched];      // prefix pages copied
            uint32_t f_full[kSched];     // full prefix pages (private pages start there)
            uint32_t f_off[kSched];      // offset of the prefix's page list
        };
        // retirement and grouping (after admission)
        struct {
            uint32_t fin[kSched];
            uint32_t fin_tokens[kSched];
            uint32_t fin_req[kSched];
            uint32_t fin_list[kSched];   // finished slots in slot order
            uint32_t key[kSched];        // grouping key per slot (prefix id + 1, 0 = none)
            uint32_t rank[kSched];       // rank among the active slots with the same key
            uint32_t kcount[kKeyTable];  // per key: slot count, then first group id
        };
    };
    uint32_t rq_head, rq_n;        // ring head at the start of admission, records read ahead
    uint32_t rq_late;              // first read-ahead record that has not arrived yet
    unsigned long long now;        // arrival clock of this pass (passes or ns since t0)
    uint32_t stop, n_fin;
    // Read ahead by load_state for the first pass after it: the tokens the
    // previous pass sampled (kAheadTokens) and the RequestRing's head and
    // tail (kAheadRing).  A persistent caller's later passes read them live.
    uint32_t tok[kSched];
    uint32_t ring_head, ring_tail, ahead;
    // this pass's admissions (full decode): slot and prefix id, for the
    // parallel page-table fill that follows the serial admission loop
    uint32_t adm_slot[kSched], adm_pfx[kSched];
    uint32_t n_adm;
    uint32_t first_sent;             // parallel admission: first stop sentinel read ahead
    uint32_t wcount[kSched / 32];    // per-warp counts (free slots, scan totals)
};
constexpr uint32_t kAheadTokens = 1u, kAheadRing = 2u;

// Admission, first part (all kSched threads): the records this pass can
// take, read ahead in one parallel round trip (nine loads per record, all
// in flight) from the RequestRing (head and tail read once) or the request
// array.  With backpressure and no free slot nothing can be admitted, and
// the source is not touched at all.
__device__ void prefetch_requests(const Dev &d, SchedShared &sh)
{
    const RtIo &io = sh.io;
    if (threadIdx.x == 0) {
        uint32_t n = 0, head;
        const uint32_t free_n = free_slot_count(sh.bitmap, d.max_slots);
        const bool can = d.drop || free_n > 0u;
        if (io.ring && (sh.ahead & kAheadRing)) {
            head = sh.ring_head;
            if (can)
                n = sh.ring_tail - head;
        } else if (io.ring) {
            head = rt_load_relaxed_u32(&io.ring->cons.head);
            if (can)
                n = rt_load_acquire_u32(&io.ring->prod.tail) - head;
        } else {
            head = sh.ctl.consumed + sh.ctl.sentinel;
            n = can && head < io.n_reqs ? io.n_reqs - head : 0u;
        }
        n = min(n, min(d.max_admit, kSched));
        if (!d.drop)
            n = min(n, free_n + 1u);  // + 1: a stop sentinel right behind them
        sh.rq_head = head;
        sh.rq_n = n;
        sh.rq_late = n;
        sh.ahead &= ~kAheadRing;
        if (io.arrivals && !io.ring)
            sh.now = io.arrival_unit == RT_ARRIVAL_NS ? rt::globaltimer_ns() - sh.ctl.t0
                                                      : sh.ctl.passes;
    }
    __syncthreads();
    if (threadIdx.x < sh.rq_n) {
        const RolloutRequest *src =
            io.ring ? &io.ring->slots[(sh.rq_head + threadIdx.x) & (REQUEST_RING_SIZE - 1)]
                    : &io.reqs[sh.rq_head + threadIdx.x];
        load_request(src, &sh.rq_buf[threadIdx.x]);
        // Arrival gate (array source): requests are taken in order, so the
        // pass may admit only those before the first one still to arrive.
        if (io.arrivals && !io.ring && io.arrivals[sh.rq_head + threadIdx.x] > sh.now)
            atomicMin(&sh.rq_late, threadIdx.x);
    }
    __syncthreads();
    if (threadIdx.x == 0)
        sh.rq_n = sh.rq_late;
    __syncthreads();
}

// Copy of a table of records as one flat array of 8-byte words, word i by
// thread i % kSched (all kSched threads call it): consecutive threads touch
// consecutive words, so every warp access is coalesced, where a record per
// thread (72 bytes apart) made each access touch 32 separate sectors.  A
// thread's words are all loaded before any is stored, so its loads are in
// flight together.
constexpr uint32_t kCopyWords = 12;  // words per thread: up to 12 x 8 x kSched bytes
__device__ __forceinline__ void copy_table(void *dst, const void *src, size_t bytes)
{
    uint64_t *d = static_cast<uint64_t *>(dst);
    const uint64_t *s = static_cast<const uint64_t *>(src);
    const size_t n = bytes / 8u;
    uint64_t v[kCopyWords];
#pragma unroll
    for (uint32_t j = 0; j < kCopyWords; j++) {
        const size_t i = threadIdx.x + (size_t)j * kSched;
        if (i < n)
            v[j] = s[i];
    }
#pragma unroll
    for (uint32_t j = 0; j < kCopyWords; j++) {
        const size_t i = threadIdx.x + (size_t)j * kSched;
        if (i < n)
            d[i] = v[j];
    }
}
static_assert(sizeof(GpuRolloutSlot) <= 8u * kCopyWords && sizeof(SlotExt) <= 8u * kCopyWords,
              "a table of kSched records fits kCopyWords words per thread");
static_assert(sizeof(GpuRolloutSlot) % 8 == 0 && sizeof(SlotExt) % 8 == 0,
              "slot records copy as whole 8-byte words");

// Load the pass state (all kSched threads).
__device__ void load_state(const Dev &d, SchedShared &sh, bool with_ext)
{
    const uint32_t s = threadIdx.x;
    // round trip 1: io block, control block, this slot's extension and the
    // token it sampled last pass
    if (s < sizeof(RtIo) / 8u)
        reinterpret_cast<uint64_t *>(&sh.io)[s] = reinterpret_cast<const uint64_t *>(d.io)[s];
    else if (s - 32u < sizeof(RtCtl) / 8u)
        reinterpret_cast<uint64_t *>(&sh.ctl)[s - 32u] = reinterpret_cast<const uint64_t *>(d.ctl)[s - 32u];
    if (with_ext) {
        copy_table(sh.ext, d.ext, (size_t)d.max_slots * sizeof(SlotExt));
        if (s < d.max_slots)
            sh.tok[s] = d.tokens[s];
    }
    __syncthreads();
    // round trip 2: the reference state table behind io.state, and the
    // RequestRing's head and tail
    GpuRolloutState *st = sh.io.state;
    copy_table(sh.slot, st->slots, (size_t)d.max_slots * sizeof(GpuRolloutSlot));
    if (s < (GPU_MAX_ROLLOUTS + 63) / 64)
        sh.bitmap[s] = st->bitmap[s];
    if (s == kSched - 1u) {
        uint32_t ahead = with_ext ? kAheadTokens : 0u;
        if (sh.io.ring) {
            sh.ring_head = rt_load_relaxed_u32(&sh.io.ring->cons.head);
            sh.ring_tail = rt_load_acquire_u32(&sh.io.ring->prod.tail);
            ahead |= kAheadRing;
        }
        sh.ahead = ahead;
    }
    __syncthreads();
}

// Store the pass state back (all kSched threads).
__device__ void store_state(const Dev &d, SchedShared &sh, bool with_ext)
{
    const uint32_t s = threadIdx.x;
    __syncthreads();
    GpuRolloutState *st = sh.io.state;
    copy_table(st->slots, sh.slot, (size_t)d.max_slots * sizeof(GpuRolloutSlot));
    if (with_ext)
        copy_table(d.ext, sh.ext, (size_t)d.max_slots * sizeof(SlotExt));
    if (s < (GPU_MAX_ROLLOUTS + 63) / 64)
        st->bitmap[s] = sh.bitmap[s];
    if (s >= 32u && s - 32u < sizeof(RtCtl) / 8u)
        reinterpret_cast<uint64_t *>(d.ctl)[s - 32u] = reinterpret_cast<const uint64_t *>(&sh.ctl)[s - 32u];
    __syncthreads();
}

// Lowest free slot below max_slots (reference find_free_slot order).
__device__ int take_lowest_free(uint64_t *bitmap, uint32_t max_slots)
{
    for (uint32_t w = 0; w < (GPU_MAX_ROLLOUTS + 63) / 64; w++) {
        uint64_t free_bits = ~bitmap[w];
        const uint32_t lo = w * 64u;
        if (lo >= max_slots)
            break;
        if (max_slots - lo < 64u)
            free_bits &= (1ull << (max_slots - lo)) - 1ull;
        if (free_bits) {
            const int b = __ffsll((long long)free_bits) - 1;
            bitmap[w] |= 1ull << b;
            return (int)(lo + (uint32_t)b);
        }
    }
    return -1;
}

// Shared-prefix groups for the attention.  Active slots decoding from the
// same prefix, in slot order, are cut into runs of up to 16; a run of one
// stays ungrouped.  Group ids: per key in key order, then run order, so the
// table is a pure function of the slot state.  All kSched threads call it.
__device__ void build_groups(const Dev &d, SchedShared &sh, uint32_t key, uint32_t shared)
{
    const uint32_t s = threadIdx.x;
    const bool table = d.max_prefixes + 1u <= kKeyTable;
    sh.key[s] = key;
    if (table)
        for (uint32_t k = s; k <= d.max_prefixes; k += kSched)
            sh.kcount[k] = 0u;
    __syncthreads();
    uint32_t rank = 0, total = 0;
    if (table) {
        // warp 0 walks the slots 32 at a time: rank = same-key slots before
        if (s < 32u) {
            for (uint32_t c = 0; c < kSched / 32u; c++) {
                const uint32_t slot = c * 32u + s;
                const uint32_t k = sh.key[slot];
                const unsigned same = __match_any_sync(0xffffffffu, k);
                const uint32_t before = (uint32_t)__popc(same & ((1u << s) - 1u));
                if (k)
                    sh.rank[slot] = sh.kcount[k] + before;
                __syncwarp();
                if (k && before == 0u)
                    sh.kcount[k] += (uint32_t)__popc(same);
                __syncwarp();
            }
        }
        __syncthreads();
        if (key) {
            rank = sh.rank[s];
            total = sh.kcount[key];
        }
        __syncthreads();
        // kcount[k] := first group id of key k (exclusive scan of group counts, warp 0)
        if (s < 32u) {
            uint32_t carry = 0;
            for (uint32_t base = 0; base <= d.max_prefixes; base += 32u) {
                const uint32_t k = base + s;
                const uint32_t n = k <= d.max_prefixes ? sh.kcount[k] : 0u;
                const uint32_t g = n / 16u + ((n % 16u) >= 2u ? 1u : 0u);
                uint32_t x = g;
#pragma unroll
                for (int o = 1; o < 32; o <<= 1) {
                    const uint32_t y = __shfl_up_sync(0xffffffffu, x, o);
                    if (s >= (uint32_t)o)
                        x += y;
                }
                if (k <= d.max_prefixes)
                    sh.kcount[k] = carry + x - g;
                carry += __shfl_sync(0xffffffffu, x, 31);
            }
            if (s == 0)
                sh.n_fin = carry;  // reused: number of groups
        }
        __syncthreads();
    } else if (key) {
        // large key spaces: scan the slots
        for (uint32_t t = 0; t < kSched; t++) {
            const uint32_t kt = sh.key[t];
            rank += (kt == key && t < s) ? 1u : 0u;
            total += kt == key ? 1u : 0u;
        }
    }
    // run r = rank / 16 of this key is a group when it has >= 2 members
    const uint32_t run = rank / 16u;
    const uint32_t run_n = min(16u, total - run * 16u);
    const bool in_group = key != 0u && run_n >= 2u;
    if (!table) {
        // group id = number of group leaders (first slot of a run of >= 2) in lower slots
        const bool leader = in_group && rank % 16u == 0u;
        const unsigned ballot = __ballot_sync(0xffffffffu, leader);
        if ((s & 31u) == 0u)
            sh.fin[s >> 5] = (uint32_t)__popc(ballot);
        __syncthreads();
        uint32_t before = 0, all = 0;
        for (uint32_t w = 0; w < kSched / 32u; w++) {
            before += w < (s >> 5) ? sh.fin[w] : 0u;
            all += sh.fin[w];
        }
        const uint32_t gid_leader = before + (uint32_t)__popc(ballot & ((1u << (s & 31u)) - 1u));
        __syncthreads();
        if (leader)
            sh.rank[s] = gid_leader;  // published for the run's members
        if (s == 0)
            sh.n_fin = all;
        __syncthreads();
    }
    uint32_t gid = 0;
    if (in_group) {
        if (table) {
            gid = sh.kcount[key] + run;
        } else {
            // the run's leader is the same-key slot of rank run * 16
            uint32_t cnt = 0;
            for (uint32_t t = 0; t <= s; t++) {
                if (sh.key[t] != key)
                    continue;
                if (cnt == run * 16u) {
                    gid = sh.rank[t];
                    break;
                }
                cnt++;
            }
        }
    }
    const bool ok = in_group && gid < d.max_groups;
    if (ok) {
        d.groups[gid].members[rank % 16u] = s;
        if (rank % 16u == 0u) {
            d.groups[gid].n_members = run_n;
            d.groups[gid].shared_pages = shared;
        }
    }
    if (s < d.max_slots) {
        d.skip[s] = ok ? shared : 0u;
        sh.ext[s].skip = ok ? shared : 0u;
    }
    __syncthreads();
    if (s == 0)
        *d.n_groups = min(sh.n_fin, d.max_groups);
}

// Admission with backpressure, all kSched threads at once (the serial loop
// below is kept for the reference's drop-when-full pacing and for traced
// runs, whose records keep their order).  The result is the serial loop's:
// requests are taken in source order, the k-th admitted one into the k-th
// lowest free slot, until a stop sentinel (consumed), max_admit, the read-
// ahead or the free slots run out.
__device__ void admit_parallel(const Dev &d, SchedShared &sh, bool full)
{
    const uint32_t s = threadIdx.x, lane = s & 31u, warp = s >> 5;
    RtCtl *ctl = &sh.ctl;
    if (s == 0)
        sh.first_sent = sh.rq_n;
    __syncthreads();
    if (s < sh.rq_n && sh.rq_buf[s].request_id == RT_REQUEST_SENTINEL)
        atomicMin(&sh.first_sent, s);
    const bool is_free =
        s < d.max_slots && ((sh.bitmap[s >> 6] >> (s & 63u)) & 1ull) == 0ull;
    const unsigned ball = __ballot_sync(0xffffffffu, is_free);
    if (lane == 0)
        sh.wcount[warp] = (uint32_t)__popc(ball);
    __syncthreads();
    uint32_t before = 0, free_n = 0;
#pragma unroll
    for (uint32_t w = 0; w < kSched / 32u; w++) {
        before += w < warp ? sh.wcount[w] : 0u;
        free_n += sh.wcount[w];
    }
    const uint32_t rank = before + (uint32_t)__popc(ball & ((1u << lane) - 1u));
    const uint32_t fs = sh.first_sent;
    const uint32_t n_adm = min(min(fs, sh.rq_n), min(free_n, d.max_admit));
    const bool take_sent = fs < sh.rq_n && n_adm == fs && fs < d.max_admit;
    const bool mine = is_free && rank < n_adm;
    if (mine) {
        const RolloutRequest rq = sh.rq_buf[rank];
        GpuRolloutSlot &rs = sh.slot[s];
        rs.active = 1u;
        rs.request_id = (uint32_t)(rq.request_id & 0xFFFFFFFFull);
        rs.tokens_generated = 0u;
        rs.max_tokens = rq.max_tokens;
        rs.kv_blocks = rq.kv_blocks;
        rs.rng_state[0] = rq.rng_seed;
        rs.rng_state[1] = rq.rng_seed ^ 0x9e3779b97f4a7c15ULL;
        rs.rng_state[2] = (rq.rng_seed << 17) ^ 0x3c6ef372fe94f82aULL;
        rs.rng_state[3] = ~rq.rng_seed;
        rs.temperature = rq.temperature;
        rs.top_k = rq.top_k;
        rs.top_p = rq.top_p;
        if (full) {
            SlotExt &e = sh.ext[s];
            const uint32_t pfx = RT_REQUEST_PREFIX(rq.request_id);
            e.row = ctl->consumed + rank;
            e.prefix = (pfx != 0u && pfx - 1u < d.max_prefixes) ? pfx : 0u;
            e.request_lo = rs.request_id;
            e.last_token = 0u;
            e.decoding = 0u;
            e.seed = rq.rng_seed;
            sh.adm_slot[rank] = s;
            sh.adm_pfx[rank] = e.prefix;
        }
    }
    const unsigned took = __ballot_sync(0xffffffffu, mine);
    if (lane == 0 && took)
        atomicOr((unsigned long long *)&sh.bitmap[warp >> 1],
                 (unsigned long long)took << (32u * (warp & 1u)));
    __syncthreads();
    if (s == 0) {
        ctl->consumed += n_adm;
        ctl->admitted += n_adm;
        if (n_adm)
            ctl->groups_ok = 0u;
        if (take_sent) {
            ctl->sentinel = 1u;
            sh.stop = 1u;
        }
        sh.n_adm = full ? n_adm : 0u;
        const uint32_t taken = n_adm + (take_sent ? 1u : 0u);
        if (sh.io.ring && taken)
            rt_store_release_u32(&sh.io.ring->cons.head, sh.rq_head + taken);
    }
    __syncthreads();
}

// The admitted slots' context and page-table rows (all kSched threads): the
// prefix's full pages first, then the slot's private pages; a partial last
// prefix page is noted for its copy on the first write.  The entries of all
// admissions form one flat range, so every load is in flight at once
// whatever the number of admissions.
__device__ void fill_admitted(const Dev &d, SchedShared &sh)
{
    const uint32_t s = threadIdx.x, lane = s & 31u, warp = s >> 5;
    const uint32_t n_adm = sh.n_adm;
    uint32_t cnt = 0;
    if (s < n_adm) {
        const uint32_t slot = sh.adm_slot[s], pfx = sh.adm_pfx[s];
        uint32_t ctx = 0, np = 0, off = 0;
        if (pfx != 0u) {
            ctx = d.pf_len[pfx - 1u];
            np = d.pf_np[pfx - 1u];
            off = d.pf_off[pfx - 1u];
        }
        // keep the context inside the page table / private pages
        const uint32_t cap = d.maxp * 16u;
        if (ctx > cap)
            ctx = cap;
        const uint32_t full_pages = ctx / 16u;
        const uint32_t n_pf = min(full_pages, np);
        // private pages fill entries full_pages .. maxp - 1, at most ppriv of them
        const uint32_t n_pv = min(d.maxp - min(full_pages, d.maxp), d.ppriv);
        cnt = n_pf + n_pv;
        sh.f_npf[s] = n_pf;
        sh.f_full[s] = full_pages;
        sh.f_off[s] = off;
        SlotExt &e = sh.ext[slot];
        e.ctx_len = ctx;
        e.pos = ctx;
        e.shared = pfx ? n_pf : 0u;
        if ((ctx & 15u) && full_pages < np) {
            e.cow_src = d.pf_pages[off + full_pages];
            e.cow_rows = ctx & 15u;
        } else {
            e.cow_src = -1;
            e.cow_rows = 0u;
        }
    }
    // exclusive prefix sum of the entry counts (n_adm <= kSched)
    uint32_t x = cnt;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= (uint32_t)o)
            x += y;
    }
    if (lane == 31u)
        sh.wcount[warp] = x;
    __syncthreads();
    uint32_t before = 0, total = 0;
#pragma unroll
    for (uint32_t w = 0; w < kSched / 32u; w++) {
        before += w < warp ? sh.wcount[w] : 0u;
        total += sh.wcount[w];
    }
    sh.f_pre[s] = before + x - cnt;
    if (s == 0)
        sh.f_pre[kSched] = total;
    __syncthreads();
    for (uint32_t e = s; e < total; e += kSched) {
        // the admission k holding entry e: largest k < n_adm with f_pre[k] <= e
        uint32_t lo = 0, hi = n_adm - 1u;
        while (lo < hi) {
            const uint32_t mid = (lo + hi + 1u) >> 1;
            if (sh.f_pre[mid] <= e)
                lo = mid;
            else
                hi = mid - 1u;
        }
        const uint32_t k = lo, j = e - sh.f_pre[k], slot = sh.adm_slot[k];
        int32_t *pt = d.page_table + (size_t)slot * d.maxp;
        const uint32_t n_pf = sh.f_npf[k];
        if (j < n_pf)
            pt[j] = d.pf_pages[sh.f_off[k] + j];
        else
            pt[sh.f_full[k] + (j - n_pf)] = d.priv[(size_t)slot * d.ppriv + (j - n_pf)];
    }
    __syncthreads();
}

// One pass of the reference rollout_worker loop (see file comment) on the
// shared-memory state.  Returns true when the loop must stop.  All kSched
// threads call it.
__device__ bool schedule_pass(const Dev &d, SchedShared &sh)
{
    const uint32_t s = threadIdx.x;
    const RtIo &io = sh.io;
    RtCtl *ctl = &sh.ctl;
    const bool full = d.decode != RT_ROLLOUT_DECODE_NONE;

    // 1. commit the tokens sampled in the previous pass
    const bool committing = full && s < d.max_slots && sh.ext[s].decoding;
    if (committing) {
        SlotExt &e = sh.ext[s];
        GpuRolloutSlot &rs = sh.slot[s];
        const uint32_t tok = (sh.ahead & kAheadTokens) ? sh.tok[s] : d.tokens[s];
        const uint32_t g = rs.tokens_generated;
        if (io.traj && e.row < io.n_rows && g < d.max_new)
            io.traj[(size_t)e.row * d.max_new + g] = tok;
        rs.tokens_generated = g + 1u;
        e.pos += 1u;
        e.last_token = tok;
        e.decoding = 0u;
    }
    if (s == 0) {
        sh.stop = 0u;
        if (ctl->passes == 0ull)
            ctl->t0 = rt::globaltimer_ns();
    }
    const uint32_t n_commit = __syncthreads_count(committing);
    if (s == 0) {
        ctl->tokens += n_commit;
        sh.ahead &= ~kAheadTokens;
    }

    // 2. admission, in source order, lowest free slot first.  The source is
    //    read ahead (prefetch_requests); a ring's head is released once.
    prefetch_requests(d, sh);
    if (!d.drop && !d.trace) {
        admit_parallel(d, sh, full);
        if (full && sh.n_adm)
            fill_admitted(d, sh);
    } else {
        if (s == 0) {
            sh.n_adm = 0u;
            uint32_t taken = 0;  // source records consumed this pass
            for (uint32_t a = 0; a < d.max_admit; a++) {
                // the read-ahead covers every record this pass can take
                if (taken >= sh.rq_n)
                    break;
                const RolloutRequest rq = sh.rq_buf[taken];
                if (rq.request_id == RT_REQUEST_SENTINEL) {
                    taken++;
                    ctl->sentinel = 1u;
                    sh.stop = 1u;
                    break;
                }
                const int slot = take_lowest_free(sh.bitmap, d.max_slots);
                if (slot < 0) {
                    if (!d.drop)
                        break;              // backpressure: leave it queued
                    taken++;                // reference: consumed and lost
                    ctl->consumed++;
                    ctl->dropped++;
                    continue;
                }
                taken++;
                const uint32_t row = ctl->consumed++;
                ctl->admitted++;
                const uint32_t rq_lo = (uint32_t)(rq.request_id & 0xFFFFFFFFull);
                trace_push(d.trace, RT_TRACE_ROLLOUT_ALLOC, rq_lo, (uint32_t)slot);
                trace_push(d.trace, RT_TRACE_DESC_CONSUMED, rq_lo, row);
                ctl->groups_ok = 0u;
                GpuRolloutSlot &rs = sh.slot[slot];
                rs.active = 1u;
                rs.request_id = (uint32_t)(rq.request_id & 0xFFFFFFFFull);
                rs.tokens_generated = 0u;
                rs.max_tokens = rq.max_tokens;
                rs.kv_blocks = rq.kv_blocks;
                rs.rng_state[0] = rq.rng_seed;
                rs.rng_state[1] = rq.rng_seed ^ 0x9e3779b97f4a7c15ULL;
                rs.rng_state[2] = (rq.rng_seed << 17) ^ 0x3c6ef372fe94f82aULL;
                rs.rng_state[3] = ~rq.rng_seed;
                rs.temperature = rq.temperature;
                rs.top_k = rq.top_k;
                rs.top_p = rq.top_p;
                if (full) {
                    // the slot's page table and context are filled in parallel below
                    SlotExt &e = sh.ext[slot];
                    const uint32_t pfx = RT_REQUEST_PREFIX(rq.request_id);
                    e.row = row;
                    e.prefix = (pfx != 0u && pfx - 1u < d.max_prefixes) ? pfx : 0u;
                    e.request_lo = rs.request_id;
                    e.last_token = 0u;
                    e.decoding = 0u;
                    e.seed = rq.rng_seed;
                    sh.adm_slot[sh.n_adm] = (uint32_t)slot;
                    sh.adm_pfx[sh.n_adm] = e.prefix;
                    sh.n_adm++;
                }
            }
            if (io.ring && taken)
                rt_store_release_u32(&io.ring->cons.head, sh.rq_head + taken);
        }
        __syncthreads();
        // Admitted slots' context and page tables, one warp per slot: the
        // prefix's pages first (up to its full pages), then the slot's private
        // pages; a partial last prefix page is copied on the first write.
        if (full) {
            const uint32_t lane = s & 31u, warp = s >> 5;
            for (uint32_t k = warp; k < sh.n_adm; k += kSched / 32u) {
                const uint32_t slot = sh.adm_slot[k], pfx = sh.adm_pfx[k];
                uint32_t ctx = 0, np = 0, off = 0;
                if (pfx != 0u) {
                    ctx = d.pf_len[pfx - 1u];
                    np = d.pf_np[pfx - 1u];
                    off = d.pf_off[pfx - 1u];
                }
                // keep the context inside the page table / private pages
                const uint32_t cap = d.maxp * 16u;
                if (ctx > cap)
                    ctx = cap;
                int32_t *pt = d.page_table + (size_t)slot * d.maxp;
                const int32_t *priv = d.priv + (size_t)slot * d.ppriv;
                const uint32_t full_pages = ctx / 16u;
                const uint32_t n_pf = min(full_pages, np);
                for (uint32_t i = lane; i < n_pf; i += 32u)
                    pt[i] = d.pf_pages[off + i];
                // private pages fill entries full_pages .. maxp - 1, at most ppriv of them
                const uint32_t n_pv = min(d.maxp - min(full_pages, d.maxp), d.ppriv);
                for (uint32_t j = lane; j < n_pv; j += 32u)
                    pt[full_pages + j] = priv[j];
                if (lane == 0) {
                    SlotExt &e = sh.ext[slot];
                    e.ctx_len = ctx;
                    e.pos = ctx;
                    e.shared = pfx ? n_pf : 0u;
                    if ((ctx & 15u) && full_pages < np) {
                        e.cow_src = d.pf_pages[off + full_pages];
                        e.cow_rows = ctx & 15u;
                    } else {
                        e.cow_src = -1;
                        e.cow_rows = 0u;
                    }
                }
            }
            __syncthreads();
        }
    }
    if (sh.stop)
        return true;  // reference: the sentinel ends the worker before the scan

    // 3. retire finished slots, in slot order
    uint32_t fin = 0;
    if (s < d.max_slots) {
        const GpuRolloutSlot &rs = sh.slot[s];
        if (rs.active && rs.tokens_generated >= rs.max_tokens) {
            fin = 1u;
            sh.fin_tokens[s] = rs.tokens_generated;
            sh.fin_req[s] = rs.request_id;
        }
    }
    sh.fin[s] = fin;
    // compact list of the finished slots, in slot order, so the serial
    // part below visits only them
    {
        const uint32_t lane = s & 31u, warp = s >> 5;
        const unsigned ball = __ballot_sync(0xffffffffu, fin != 0u);
        if (lane == 0)
            sh.wcount[warp] = (uint32_t)__popc(ball);
        __syncthreads();
        uint32_t before = 0;
#pragma unroll
        for (uint32_t w = 0; w < kSched / 32u; w++)
            before += w < warp ? sh.wcount[w] : 0u;
        if (fin)
            sh.fin_list[before + (uint32_t)__popc(ball & ((1u << lane) - 1u))] = s;
    }
    const uint32_t n_fin = __syncthreads_count(fin);
    if (n_fin && s == 0)
        ctl->groups_ok = 0u;
    if (n_fin && s == 0) {
        // a DoneRing takes the batch with one head read and one tail release
        // while it has room (done_ring_push per record otherwise)
        uint32_t dn_tail = 0, dn_room = 0, dn_pushed = 0;
        if (io.done_ring) {
            const uint32_t head = rt_load_acquire_u32(&io.done_ring->cons.head);
            dn_tail = rt_load_relaxed_u32(&io.done_ring->prod.tail);
            dn_room = (uint32_t)REQUEST_RING_SIZE - (dn_tail - head);
        }
        for (uint32_t j = 0; j < n_fin; j++) {
            const uint32_t k = sh.fin_list[j];
            RolloutDone rec;
            rec.request_id = sh.fin_req[k];
            rec.rollout_id = k;
            rec.tokens_generated = sh.fin_tokens[k];
            rec.reward = reward_for(d, sh.fin_req[k], sh.fin_tokens[k]);
            rec.status = 0u;
            trace_push(d.trace, RT_TRACE_REWARD_POSTED, sh.fin_req[k], sh.fin_tokens[k]);
            trace_push(d.trace, RT_TRACE_TRAJECTORY_DONE, sh.fin_req[k], sh.fin_tokens[k]);
            trace_push(d.trace, RT_TRACE_ROLLOUT_FREE, sh.fin_req[k], k);
            if (io.done_ring && dn_room) {
                uint64_t *dst = reinterpret_cast<uint64_t *>(
                    &io.done_ring->slots[(dn_tail + dn_pushed) & (REQUEST_RING_SIZE - 1)]);
                const uint64_t *src = reinterpret_cast<const uint64_t *>(&rec);
                st_sys_u64(dst, src[0]);
                st_sys_u64(dst + 1, src[1]);
                st_sys_u64(dst + 2, src[2]);
                dn_pushed++;
                dn_room--;
                ctl->done++;
                continue;
            }
            if (dn_pushed) {  // publish the batch before the slow path
                rt_store_release_u32(&io.done_ring->prod.tail, dn_tail + dn_pushed);
                dn_tail += dn_pushed;
                dn_pushed = 0;
            }
            if (!sink_push(io, ctl, rec)) {
                ctl->error = RT_ETIMEOUT;
                sh.stop = 1u;
                break;
            }
            ctl->done++;
        }
        if (dn_pushed)
            rt_store_release_u32(&io.done_ring->prod.tail, dn_tail + dn_pushed);
        if (io.step_count)
            atomicAdd(io.step_count, (unsigned long long)n_fin);
    }
    __syncthreads();
    if (fin) {
        GpuRolloutSlot &rs = sh.slot[s];
        rs.active = 0u;
        atomicAnd((unsigned long long *)&sh.bitmap[s / 64u], ~(1ull << (s % 64u)));
        if (io.rewards && full && sh.ext[s].row < io.n_rows)
            io.rewards[sh.ext[s].row] = reward_for(d, sh.fin_req[s], sh.fin_tokens[s]);
    }
    if (sh.stop)
        return true;

    // 4. this pass's decode: every slot still active generates one token
    uint32_t act = 0;
    int32_t my_len = 0;  // the slot's attention length this pass
    if (s < d.max_slots) {
        GpuRolloutSlot &rs = sh.slot[s];
        act = rs.active && !fin;
        if (full) {
            SlotExt &e = sh.ext[s];
            const bool room = e.pos < d.maxp * 16u;
            if (act && !room) {
                act = 0u;  // context full: counts as an error, slot is left idle
                atomicCAS(&ctl->error, 0, RT_EDEVICE);
            }
            d.enable[s] = act;
            my_len = act ? (int32_t)(e.pos + 1u) : 0;
            d.seq_lens[s] = my_len;
            if (act) {
                e.decoding = 1u;
                rt_sample_row_t r;
                r.temperature = rs.temperature;
                r.top_k = rs.top_k;
                r.top_p = rs.top_p;
                r.rollout_id = e.request_lo;
                r.step = rs.tokens_generated;
                r.seed = e.seed;
                d.srows[s] = r;
            }
        } else if (act) {
            rs.tokens_generated++;  // the reference's counter-only decode
        }
    }
    const uint32_t n_act = __syncthreads_count(act);
    // The group table depends only on which slots are active (and their
    // prefixes): rebuild it when a slot was admitted or retired, or when the
    // active count changed for another reason (a slot whose context is full).
    if (full && d.max_groups && !(ctl->groups_ok && ctl->groups_act == n_act)) {
        const bool key_ok = act && sh.ext[s].prefix != 0u && sh.ext[s].shared != 0u;
        build_groups(d, sh, key_ok ? sh.ext[s].prefix : 0u, key_ok ? sh.ext[s].shared : 0u);
        if (s == 0) {
            ctl->groups_ok = 1u;
            ctl->groups_act = n_act;
        }
    }
    if (full && d.attn_chunks) {
        // This pass's attention items (rt::attn_seq_shape of every slot), for
        // the attention launch: the largest chunk count (at least 1: chunk 0
        // of every slot) and the slots' full chunks (all but chunk 0) as an
        // exclusive prefix over slots, so that it hands out no empty items.
        uint32_t nch = 0;
        if (s < d.max_slots && my_len > 0) {
            const uint32_t skip = d.max_groups ? sh.ext[s].skip : 0u;
            const rt::AttnSeqShape shp = rt::attn_seq_shape(my_len, skip, d.maxp * 16u, d.maxp,
                                                            d.attn_gcp, d.attn_mg, d.attn_cp);
            nch = (uint32_t)shp.n_chunks;
        }
        const uint32_t lane = s & 31u, warp = s >> 5;
        const uint32_t fulls = nch > 1u ? nch - 1u : 0u;
        uint32_t incl = fulls;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= (uint32_t)o)
                incl += y;
        }
        const uint32_t wmax = __reduce_max_sync(0xffffffffu, nch);
        if (lane == 31u)
            sh.wcount[warp] = incl;
        __syncthreads();
        uint32_t before = 0, total = 0;
        for (uint32_t w = 0; w < kSched / 32u; w++) {
            before += w < warp ? sh.wcount[w] : 0u;
            total += sh.wcount[w];
        }
        __syncthreads();
        if (lane == 0u)
            sh.wcount[warp] = wmax;
        __syncthreads();
        uint32_t m = 1u;
        for (uint32_t w = 0; w < kSched / 32u; w++)
            m = max(m, sh.wcount[w]);
        if (s < d.max_slots)
            d.attn_chunks[2u + s] = before + incl - fulls;
        if (s == 0) {
            d.attn_chunks[0] = m;
            d.attn_chunks[1] = total;
        }
    }

    // 5. loop control
    if (s == 0) {
        trace_push(d.trace, RT_TRACE_DECODE_BATCH, n_act, (uint32_t)ctl->passes);
        ctl->passes++;
        if (!full)
            ctl->tokens += n_act;  // full decode counts tokens when they are committed
        if (n_act > ctl->max_active)
            ctl->max_active = n_act;
        bool stop = ctl->error != 0;
        if (n_act == 0u && !io.ring && src_empty(io, ctl))
            stop = true;
        if (n_act == 0u && io.ring && src_empty(io, ctl)) {
            const uint64_t now = rt::globaltimer_ns();
            if (ctl->idle_since == 0ull)
                ctl->idle_since = now;
            else if (now - ctl->idle_since > d.idle_ns) {
                ctl->error = RT_ETIMEOUT;
                stop = true;
            }
        } else {
            ctl->idle_since = 0ull;
        }
        if (ctl->passes >= d.max_passes) {
            ctl->error = RT_ETIMEOUT;
            stop = true;
        }
        sh.stop = stop ? 1u : 0u;
    }
    __syncthreads();
    return sh.stop != 0u;
}

__global__ void __launch_bounds__(kSched, 1)
schedule_kernel(const Dev d, cudaGraphConditionalHandle handle, int in_graph)
{
    __shared__ SchedShared sh;
    const bool full = d.decode != RT_ROLLOUT_DECODE_NONE;
    // Inside the graph loop this kernel is a programmatic dependent of the
    // previous pass's sampler: wait for its tokens before reading anything
    // (a no-op for an ordinary launch).
    rt::grid_dep_wait();
    // The prepare kernel (a programmatic dependent launch) may be scheduled
    // now; it waits for this kernel to complete before reading its outputs.
    rt::grid_dep_launch();
    load_state(d, sh, full);
    if (sh.ctl.stop) {
        // An earlier pass of this graph iteration ended the loop (the body
        // holds several passes): run nothing.  That pass left every slot
        // disabled, so this pass's decode chain is a no-op too.
        if (threadIdx.x == 0 && in_graph)
            cudaGraphSetConditional(handle, 0u);
        return;
    }
    const bool stop = schedule_pass(d, sh);
    if (stop) {
        // The decode chain of this pass still runs: make it a no-op.
        const uint32_t s = threadIdx.x;
        if (s == 0)
            sh.ctl.stop = 1u;
        if (s < d.max_slots) {
            d.enable[s] = 0u;
            if (d.seq_lens)
                d.seq_lens[s] = 0;
        }
        if (s == 0 && d.max_groups) {
            *d.n_groups = 0u;
            sh.ctl.groups_ok = 0u;
        }
    }
    store_state(d, sh, full);
    if (threadIdx.x == 0 && in_graph)
        cudaGraphSetConditional(handle, stop ? 0u : 1u);
}

// First write into a shared prefix's partial page: the slot's private copy
// (one CTA; the copy is complete when this returns).
__device__ __forceinline__ void cow_copy(const Dev &d, SlotExt &e, const int32_t *pt, int32_t cow)
{
    if (cow >= 0) {
        const uint64_t page_elems = rt_page_bytes(d.hkv) / 2u;
        const uint4 *src = reinterpret_cast<const uint4 *>(d.arena + (uint64_t)cow * page_elems);
        uint4 *dst = reinterpret_cast<uint4 *>(d.arena + (uint64_t)pt[e.ctx_len >> 4] * page_elems);
        const uint32_t n16 = (uint32_t)(rt_page_bytes(d.hkv) / 16u);
        for (uint32_t i = threadIdx.x; i < n16; i += blockDim.x)
            dst[i] = src[i];
        __syncthreads();
        if (threadIdx.x == 0)
            e.cow_src = -1;
    }
}

__global__ void __launch_bounds__(256) prepare_kernel(const Dev d)
{
    const uint32_t s = blockIdx.x;
    rt::grid_dep_wait();    // the schedule kernel's plan is complete
    rt::grid_dep_launch();  // the attention kernels may be scheduled
    // the slot's flag and its extension in one round trip
    SlotExt &e = d.ext[s];
    const uint32_t en = d.enable[s];
    const uint32_t pos = e.pos, lt = e.last_token, rq = e.request_lo;
    const uint64_t seed = e.seed;
    const int32_t cow = e.cow_src;
    if (!en)
        return;
    const int32_t *pt = d.page_table + (size_t)s * d.maxp;
    const uint64_t page = (uint64_t)pt[pos >> 4];
    cow_copy(d, e, pt, cow);
    const uint32_t row = pos & 15u;
    // new token's K and V: hkv heads x 2 planes x 128 dims, 4 per Philox block
    for (uint32_t g = threadIdx.x; g < d.hkv * 2u * 32u; g += blockDim.x) {
        const uint32_t h = g >> 6, plane = (g >> 5) & 1u, d4 = g & 31u;
        float z[4];
        rt::philox_normal4(seed, pos, rq, 0x6B000000u | (plane << 8) | h, z, (lt << 5) | d4);
        __nv_bfloat16 *dst = d.arena + rt_page_elem_offset(page, h, plane, row, d.hkv) + d4 * 4u;
        reinterpret_cast<uint2 *>(dst)[0] =
            make_uint2(rt::pack_bf16x2(z[0], z[1]), rt::pack_bf16x2(z[2], z[3]));
    }
    // query: hq heads x 128 dims
    for (uint32_t g = threadIdx.x; g < d.hq * 32u; g += blockDim.x) {
        const uint32_t h = g >> 5, d4 = g & 31u;
        float z[4];
        rt::philox_normal4(seed, pos, rq, 0x71000000u | h, z, (lt << 5) | d4);
        __nv_bfloat16 *dst = d.q + ((size_t)s * d.hq + h) * 128u + d4 * 4u;
        reinterpret_cast<uint2 *>(dst)[0] =
            make_uint2(rt::pack_bf16x2(z[0], z[1]), rt::pack_bf16x2(z[2], z[3]));
    }
}

// ---- model decode: embedding gather, q / K / V from the QKV projection,
// attention output to bf16 (the projections themselves are rt_gemm_bf16)

// x_s = embed[last token of slot s] (token 0 before the slot's first token).
__global__ void __launch_bounds__(256) embed_kernel(const Dev d)
{
    const uint32_t s = blockIdx.x;
    rt::grid_dep_wait();  // the schedule kernel's plan is complete
    rt::grid_dep_launch();
    if (!d.enable[s])
        return;
    const uint32_t tok = min(d.ext[s].last_token, d.vocab - 1u);
    if (threadIdx.x == 0)
        d.emb_tok[s] = tok;
    const uint4 *src = reinterpret_cast<const uint4 *>(d.w_embed + (size_t)tok * d.dm);
    uint4 *dst = reinterpret_cast<uint4 *>(d.hin + (size_t)s * d.dm);
    for (uint32_t i = threadIdx.x; i < d.dm / 8u; i += blockDim.x)
        dst[i] = __ldg(src + i);
}

// The slot's copy-on-write page, then q (bf16) and the new token's K and V
// (bf16, into its page row) from the fp32 QKV projection.
__global__ void __launch_bounds__(256) model_prepare_kernel(const Dev d)
{
    const uint32_t s = blockIdx.x;
    rt::grid_dep_wait();  // the QKV projection is complete
    rt::grid_dep_launch();
    SlotExt &e = d.ext[s];
    const uint32_t en = d.enable[s];
    const int32_t cow = e.cow_src;
    if (!en)
        return;
    const int32_t *pt = d.page_table + (size_t)s * d.maxp;
    cow_copy(d, e, pt, cow);
    const float4 *row = reinterpret_cast<const float4 *>(d.qkv + (size_t)s * d.qkv_n);
    const uint32_t nq4 = d.hq * 32u;  // q: hq heads x 128 dims, 4 per float4
    for (uint32_t g = threadIdx.x; g < nq4; g += blockDim.x) {
        const float4 v = row[g];
        reinterpret_cast<uint2 *>(d.q + (size_t)s * d.hq * 128u)[g] =
            make_uint2(rt::pack_bf16x2(v.x, v.y), rt::pack_bf16x2(v.z, v.w));
    }
    const uint32_t pos = e.pos;
    const uint64_t page = (uint64_t)pt[pos >> 4];
    const uint32_t prow = pos & 15u;
    for (uint32_t g = threadIdx.x; g < d.hkv * 2u * 32u; g += blockDim.x) {
        const uint32_t plane = g / (d.hkv * 32u), h = (g >> 5) % d.hkv, d4 = g & 31u;
        const float4 v = row[nq4 + g];  // k rows of every kv head, then v rows
        __nv_bfloat16 *dst = d.arena + rt_page_elem_offset(page, h, plane, prow, d.hkv) + d4 * 4u;
        reinterpret_cast<uint2 *>(dst)[0] =
            make_uint2(rt::pack_bf16x2(v.x, v.y), rt::pack_bf16x2(v.z, v.w));
    }
}

// hidden_out = bf16(attention output), the LM head's input.
__global__ void __launch_bounds__(256) hidden_kernel(const Dev d)
{
    const uint32_t s = blockIdx.x;
    rt::grid_dep_wait();  // the attention is complete
    if (d.enable[s]) {
        const float4 *src = reinterpret_cast<const float4 *>(d.attn_out + (size_t)s * d.dm);
        uint2 *dst = reinterpret_cast<uint2 *>(d.hout + (size_t)s * d.dm);
        for (uint32_t i = threadIdx.x; i < d.dm / 4u; i += blockDim.x) {
            const float4 v = src[i];
            dst[i] = make_uint2(rt::pack_bf16x2(v.x, v.y), rt::pack_bf16x2(v.z, v.w));
        }
    }
    rt::grid_dep_launch();
}

// ---- model prefill of a registered prefix (rt_rollout_prefill) ----

// x_i = embed[tokens[i]] for the chunk's tokens (one CTA per token).
__global__ void __launch_bounds__(256) prefill_embed_kernel(const uint32_t *tokens,
                                                            const __nv_bfloat16 *embed,
                                                            __nv_bfloat16 *x, uint32_t dm,
                                                            uint32_t vocab, int32_t *error)
{
    const uint32_t i = blockIdx.x;
    uint32_t tok = tokens[i];
    if (tok >= vocab) {
        if (threadIdx.x == 0)
            atomicCAS(error, 0, RT_EDEVICE);
        tok = 0u;
    }
    const uint4 *src = reinterpret_cast<const uint4 *>(embed + (size_t)tok * dm);
    uint4 *dst = reinterpret_cast<uint4 *>(x + (size_t)i * dm);
    for (uint32_t j = threadIdx.x; j < dm / 8u; j += blockDim.x)
        dst[j] = __ldg(src + j);
}

// K and V rows of token (first + i) (fp32 projection [k heads | v heads] x
// 128) into the prefix page holding that position, as bf16.
__global__ void __launch_bounds__(256) prefill_scatter_kernel(const float *kv, const int32_t *pages,
                                                              uint32_t first, uint32_t hkv,
                                                              __nv_bfloat16 *arena)
{
    const uint32_t i = blockIdx.x, pos = first + i;
    const uint64_t page = (uint64_t)pages[pos >> 4];
    const uint32_t prow = pos & 15u;
    const float4 *row = reinterpret_cast<const float4 *>(kv + (size_t)i * hkv * 256u);
    for (uint32_t g = threadIdx.x; g < hkv * 2u * 32u; g += blockDim.x) {
        const uint32_t plane = g / (hkv * 32u), h = (g >> 5) % hkv, d4 = g & 31u;
        const float4 v = row[g];
        __nv_bfloat16 *dst = arena + rt_page_elem_offset(page, h, plane, prow, hkv) + d4 * 4u;
        reinterpret_cast<uint2 *>(dst)[0] =
            make_uint2(rt::pack_bf16x2(v.x, v.y), rt::pack_bf16x2(v.z, v.w));
    }
}

// logits[v] = std * N(0,1), Philox key = seed, counter = (token index lo,
// request low 32, tag | token index hi, v / 4).  With cmax, also each
// 16-column chunk's maximum (rt_logits_chunk_max's layout) for the sampler.
// A warp walks 32 consecutive 4-column groups at a time (start - lane is its
// first group; blockDim and stride are multiples of 32), so the four groups
// of a chunk sit in four adjacent lanes and meet with two shuffles.
__device__ __forceinline__ void logits_row(float *out, float *cmax, uint32_t vocab,
                                           uint64_t seed, uint32_t request_lo, uint64_t tix,
                                           float stdv, uint32_t start, uint32_t stride)
{
    const uint32_t groups = (vocab + 3u) / 4u;
    const uint32_t lane = threadIdx.x & 31u;
    for (uint32_t g0 = start - lane; g0 < groups; g0 += stride) {
        const uint32_t g = g0 + lane;
        float m = -INFINITY;
        if (g < groups) {
            float z[4];
            rt::philox_normal4(seed, (uint32_t)tix, request_lo,
                               0x4C000000u | (uint32_t)((tix >> 32) & 0xFFFFu), z, g);
            const uint32_t v = g * 4u;
            const float x[4] = {stdv * z[0], stdv * z[1], stdv * z[2], stdv * z[3]};
            if (v + 3u < vocab && ((reinterpret_cast<uintptr_t>(out + v) & 15u) == 0u)) {
                reinterpret_cast<float4 *>(out + v)[0] = make_float4(x[0], x[1], x[2], x[3]);
                m = rt::nan_max(rt::nan_max(x[0], x[1]), rt::nan_max(x[2], x[3]));
            } else {
                for (uint32_t k = 0; k < 4u && v + k < vocab; k++) {
                    out[v + k] = x[k];
                    m = rt::nan_max(m, x[k]);
                }
            }
        }
        if (cmax) {
            m = rt::nan_max(m, __shfl_xor_sync(0xffffffffu, m, 1));
            m = rt::nan_max(m, __shfl_xor_sync(0xffffffffu, m, 2));
            if ((g & 3u) == 0u && g < groups)
                cmax[g / 4u] = m;
        }
    }
}

__global__ void __launch_bounds__(256) logits_kernel(const Dev d)
{
    const uint32_t s = blockIdx.y;
    rt::grid_dep_wait();  // launched as a programmatic dependent of the attention
    if (d.enable[s]) {
        const rt_sample_row_t r = d.srows[s];
        logits_row(d.logits + (size_t)s * d.vocab, d.cmax + (size_t)s * d.cstride, d.vocab,
                   r.seed, r.rollout_id, r.step, d.logit_std, blockIdx.x * blockDim.x + threadIdx.x,
                   gridDim.x * blockDim.x);
    }
    // The sampler may be scheduled once every CTA has written its logits.
    rt::grid_dep_launch();
}

// Launch as a programmatic dependent of the previous kernel in the stream.
template <typename... Args>
cudaError_t launch_pdl(void (*kernel)(Args...), dim3 grid, dim3 block, cudaStream_t st,
                       const Args &...args)
{
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = 0;
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, args...);
}

__global__ void logits_synth_kernel(float *out, uint32_t vocab, uint64_t seed, uint32_t rq,
                                    uint64_t tix, float stdv)
{
    logits_row(out, nullptr, vocab, seed, rq, tix, stdv, blockIdx.x * blockDim.x + threadIdx.x,
               gridDim.x * blockDim.x);
}

// Persistent single-CTA worker: the reference's pass loop, counter-only.
// The state table stays in shared memory for the whole run and is stored
// back when the loop ends.
__global__ void __launch_bounds__(kSched, 1) persistent_worker_kernel(const Dev d)
{
    __shared__ SchedShared sh;
    load_state(d, sh, false);
    for (;;) {
        if (schedule_pass(d, sh))
            break;
        if (threadIdx.x == 0 && sh.ctl.idle_since != 0ull)
            __nanosleep(1000);
        __syncthreads();
    }
    if (threadIdx.x == 0)
        sh.ctl.stop = 1u;
    store_state(d, sh, false);
}

template <typename T>
cudaError_t dalloc(T **p, size_t count)
{
    return cudaMalloc(reinterpret_cast<void **>(p), count * sizeof(T) + 16);
}

}  // namespace

// ------------------------------------------------------------------- engine
struct rt_rollout {
    rt_rollout_config_t cfg;
    Dev d;
    KVArena *arena;
    int64_t *priv_blocks;  // host list of reserved arena blocks (released on destroy)
    uint32_t n_priv;
    rt_attn_params_t ap;
    rt_attn_group_params_t gp;
    void *attn_ws;
    size_t attn_ws_bytes;
    uint32_t pf_used;
    int device;
    cudaStream_t cap;
    cudaGraph_t graph;
    cudaGraphExec_t exec;
    RtIo *io_stage;  // pinned host staging of the io block
    // registered prefixes (host copies): token length and page-list offset
    uint32_t *pf_len_h, *pf_off_h;
    // model prefill scratch: embeddings and K/V projections of a token chunk
    __nv_bfloat16 *pre_x;
    float *pre_kv;
    // model decode: the QKV projection through cuBLAS, with its own workspace
    // (set once, so that calls inside stream capture allocate nothing)
    cublasHandle_t blas;
    void *blas_ws;
};

namespace {

// The decode chain of one pass (after the schedule kernel).  When `ev` is
// given, events are recorded around each of the four launches.
// K-splits that fill the GPU for an M x N projection (each split >= 4
// K-slices of 64).
uint32_t gemm_splits(uint32_t M, uint32_t N, uint32_t K)
{
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const uint32_t units = ((M + 255u) / 256u) * ((N + 223u) / 224u);
    const uint32_t by_sm = (uint32_t)sms / units;
    return std::max(1u, std::min(by_sm, K / 256u));
}

// qkv fp32 [slots][qkv_n] = hin bf16 [slots][dm] x w_qkv bf16 [qkv_n][dm]^T.
// A plain GEMM of a narrow shape (N = 6,144): cuBLAS takes it in ~15 us
// where the tcgen05 kernel of gemm.cu, built for the LM head's wide N, needs
// K-splits and a reduction (~27 us).  Row-major C = A B^T is the
// column-major C^T = B A^T that cuBLAS computes.
int qkv_projection(rt_rollout *e, cudaStream_t st)
{
    const Dev &d = e->d;
    const float one = 1.0f, zero = 0.0f;
    cublasStatus_t bs = cublasSetStream(e->blas, st);
    if (bs == CUBLAS_STATUS_SUCCESS)
        bs = cublasGemmEx(e->blas, CUBLAS_OP_T, CUBLAS_OP_N, (int)d.qkv_n, (int)d.max_slots,
                          (int)d.dm, &one, d.w_qkv, CUDA_R_16BF, (int)d.dm, d.hin, CUDA_R_16BF,
                          (int)d.dm, &zero, d.qkv, CUDA_R_32F, (int)d.qkv_n, CUBLAS_COMPUTE_32F,
                          CUBLAS_GEMM_DEFAULT);
    if (bs != CUBLAS_STATUS_SUCCESS) {
        rt::set_error("rollout: QKV projection (cuBLAS status %d)", (int)bs);
        return RT_ECUDA;
    }
    return RT_OK;
}

int launch_decode_model(rt_rollout *e, cudaStream_t st, cudaEvent_t *ev)
{
    const Dev &d = e->d;
    if (ev)
        cudaEventRecord(ev[0], st);
    cudaError_t err = launch_pdl(embed_kernel, dim3(d.max_slots), dim3(256), st, d);
    if (err != cudaSuccess)
        return rt::cuda_fail(err, "rollout: embed launch");
    int rc = qkv_projection(e, st);
    if (rc != RT_OK)
        return rc;
    err = launch_pdl(model_prepare_kernel, dim3(d.max_slots), dim3(256), st, d);
    if (err != cudaSuccess)
        return rt::cuda_fail(err, "rollout: model prepare launch");
    if (ev)
        cudaEventRecord(ev[1], st);
    rc = d.max_groups
             ? rt::attn_launch(&e->ap, &e->gp, d.q, d.arena, d.page_table, d.seq_lens, d.groups,
                               d.n_groups, d.skip, d.attn_out, e->attn_ws, e->attn_ws_bytes,
                               d.attn_chunks, st)
             : rt::attn_launch(&e->ap, nullptr, d.q, d.arena, d.page_table, d.seq_lens, nullptr,
                               nullptr, nullptr, d.attn_out, e->attn_ws, e->attn_ws_bytes,
                               d.attn_chunks, st);
    if (rc != RT_OK)
        return rc;
    if (ev)
        cudaEventRecord(ev[2], st);
    err = launch_pdl(hidden_kernel, dim3(d.max_slots), dim3(256), st, d);
    if (err != cudaSuccess)
        return rt::cuda_fail(err, "rollout: hidden launch");
    rt_gemm_params_t gl = {d.max_slots, d.vocab, d.dm, d.dm, d.dm, d.vocab, d.split_lm, 0u};
    // the LM head's epilogue also writes each row's 16-column maxima for the sampler
    rc = rt_gemm_bf16_chunk_max(&gl, d.hout, d.w_lm, d.logits, d.gemm_ws, d.gemm_ws_bytes,
                                d.gemm_err, d.cmax, d.cstride, st);
    if (rc != RT_OK)
        return rc;
    if (ev)
        cudaEventRecord(ev[3], st);
    rt_sample_params_t sp;
    sp.num_rows = d.max_slots;
    sp.vocab = d.vocab;
    sp.row_stride = d.vocab;
    sp.fused_cum = 1u;
    sp.row_enable = d.enable;
    rc = rt::sample_rows_launch(&sp, d.logits, d.srows, d.tokens, st, true, d.cmax, d.cstride);
    if (ev)
        cudaEventRecord(ev[4], st);
    return rc;
}

int launch_decode(rt_rollout *e, cudaStream_t st, cudaEvent_t *ev)
{
    const Dev &d = e->d;
    if (d.decode == RT_ROLLOUT_DECODE_MODEL)
        return launch_decode_model(e, st, ev);
    if (ev)
        cudaEventRecord(ev[0], st);
    // Every kernel of the chain is a programmatic dependent launch: it may be
    // scheduled while its predecessor finishes and waits for it on the GPU.
    cudaError_t err = launch_pdl(prepare_kernel, dim3(d.max_slots), dim3(256), st, d);
    if (err != cudaSuccess)
        return rt::cuda_fail(err, "rollout: prepare launch");
    if (ev)
        cudaEventRecord(ev[1], st);
    int rc = d.max_groups
                 ? rt::attn_launch(&e->ap, &e->gp, d.q, d.arena, d.page_table, d.seq_lens,
                                   d.groups, d.n_groups, d.skip, d.attn_out, e->attn_ws,
                                   e->attn_ws_bytes, d.attn_chunks, st)
                 : rt::attn_launch(&e->ap, nullptr, d.q, d.arena, d.page_table, d.seq_lens,
                                   nullptr, nullptr, nullptr, d.attn_out, e->attn_ws,
                                   e->attn_ws_bytes, d.attn_chunks, st);
    if (rc != RT_OK)
        return rc;
    if (ev)
        cudaEventRecord(ev[2], st);
    const dim3 lg((d.vocab / 4u + 1023u) / 1024u, d.max_slots);
    err = launch_pdl(logits_kernel, lg, dim3(256), st, d);
    if (err != cudaSuccess)
        return rt::cuda_fail(err, "rollout: logits launch");
    if (ev)
        cudaEventRecord(ev[3], st);
    rt_sample_params_t sp;
    sp.num_rows = d.max_slots;
    sp.vocab = d.vocab;
    sp.row_stride = d.vocab;
    sp.fused_cum = 1u;
    sp.row_enable = d.enable;
    // the logits kernel wrote each row's 16-column maxima beside it
    rc = rt::sample_rows_launch(&sp, d.logits, d.srows, d.tokens, st, true, d.cmax, d.cstride);
    if (ev)
        cudaEventRecord(ev[4], st);
    return rc;
}

int engine_build_graph(rt_rollout *e)
{
    cudaError_t err;
    cudaGraphConditionalHandle h;
    if ((err = cudaGraphCreate(&e->graph, 0)) != cudaSuccess)
        return rt::cuda_fail(err, "rollout: cudaGraphCreate");
    if ((err = cudaGraphConditionalHandleCreate(&h, e->graph, 1, cudaGraphCondAssignDefault)) !=
        cudaSuccess)
        return rt::cuda_fail(err, "rollout: cudaGraphConditionalHandleCreate");
    // cudaGraphNodeParams has no default constructor in C++: zeroed storage
    alignas(cudaGraphNodeParams) unsigned char storage[sizeof(cudaGraphNodeParams)];
    memset(storage, 0, sizeof(storage));
    cudaGraphNodeParams &cp = *reinterpret_cast<cudaGraphNodeParams *>(storage);
    cp.type = cudaGraphNodeTypeConditional;
    cp.conditional.handle = h;
    cp.conditional.type = cudaGraphCondTypeWhile;
    cp.conditional.size = 1;
    cudaGraphNode_t node;
    if ((err = cudaGraphAddNode(&node, e->graph, nullptr, 0, &cp)) != cudaSuccess)
        return rt::cuda_fail(err, "rollout: cudaGraphAddNode(conditional)");
    cudaGraph_t body = cp.conditional.phGraph_out[0];
    // The body holds kPassesPerIteration passes: every iteration of a
    // conditional WHILE node costs several microseconds of relaunch on top
    // of the kernels' own boundaries, so one iteration per pass would add it
    // to every token.  A pass after the one that stopped the loop does
    // nothing (schedule_kernel returns at once, the decode chain finds every
    // slot disabled).

    if ((err = cudaStreamBeginCaptureToGraph(e->cap, body, nullptr, nullptr, 0,
                                             cudaStreamCaptureModeThreadLocal)) != cudaSuccess)
        return rt::cuda_fail(err, "rollout: cudaStreamBeginCaptureToGraph");
    int rc = RT_OK;
    const Dev &d = e->d;
    for (int k = 0; k < kPassesPerIteration && rc == RT_OK; k++) {
        // after the first, each pass's schedule kernel is a programmatic
        // dependent of the previous pass's sampler
        if (k == 0 || e->cfg.decode_mode == RT_ROLLOUT_DECODE_NONE)
            schedule_kernel<<<1, kSched, 0, e->cap>>>(d, h, 1);
        else if ((err = launch_pdl(schedule_kernel, dim3(1), dim3(kSched), e->cap, d, h, 1)) !=
                 cudaSuccess)
            rc = rt::cuda_fail(err, "rollout: schedule launch");
        if (rc != RT_OK)
            break;
        if (e->cfg.decode_mode != RT_ROLLOUT_DECODE_NONE)
            rc = launch_decode(e, e->cap, nullptr);
    }
    cudaGraph_t captured = nullptr;
    err = cudaStreamEndCapture(e->cap, &captured);
    if (rc != RT_OK)
        return rc;
    if (err != cudaSuccess)
        return rt::cuda_fail(err, "rollout: cudaStreamEndCapture");
    if ((err = cudaGraphInstantiate(&e->exec, e->graph, 0)) != cudaSuccess)
        return rt::cuda_fail(err, "rollout: cudaGraphInstantiate");
    return RT_OK;
}

void engine_free(rt_rollout *e)
{
    if (!e)
        return;
    if (e->exec)
        cudaGraphExecDestroy(e->exec);
    if (e->graph)
        cudaGraphDestroy(e->graph);
    if (e->cap)
        cudaStreamDestroy(e->cap);
    void *bufs[] = {e->d.io, e->d.ctl, e->d.ext, e->d.page_table, e->d.priv, e->d.seq_lens,
                    e->d.enable, e->d.srows, e->d.tokens, e->d.q, e->d.attn_out, e->d.logits,
                    e->d.cmax, e->d.attn_chunks, e->d.pf_len, e->d.pf_np, e->d.pf_off, e->d.pf_pages, e->d.groups,
                    e->d.n_groups, e->d.skip, e->attn_ws, e->d.hin, e->d.hout, e->d.qkv,
                    e->d.emb_tok, e->d.gemm_err, e->d.gemm_ws, e->pre_x, e->pre_kv};
    for (void *p : bufs)
        if (p)
            cudaFree(p);
    if (e->io_stage)
        cudaFreeHost(e->io_stage);
    if (e->blas)
        cublasDestroy(e->blas);
    if (e->blas_ws)
        cudaFree(e->blas_ws);
    if (e->arena && e->priv_blocks)
        for (uint32_t i = 0; i < e->n_priv; i++)
            arena_release(e->arena, e->priv_blocks[i]);
    free(e->priv_blocks);
    delete[] e->pf_len_h;
    delete[] e->pf_off_h;
    delete e;
}

}  // namespace

static uint32_t npf_h(const rt_rollout_config_t *cfg)
{
    return cfg->max_prefixes ? cfg->max_prefixes : 1u;
}

extern "C" int rt_rollout_create(const rt_rollout_config_t *cfg, KVArena *arena, rt_rollout_t **out)
{
    if (!cfg || !out) {
        rt::set_error("rollout: null argument");
        return RT_EINVAL;
    }
    *out = nullptr;
    const bool full = cfg->decode_mode != RT_ROLLOUT_DECODE_NONE;
    if (cfg->max_slots == 0 || cfg->max_slots > GPU_MAX_ROLLOUTS || cfg->max_admit == 0 ||
        cfg->decode_mode > RT_ROLLOUT_DECODE_MODEL) {
        rt::set_error("rollout: max_slots 1..%d, max_admit >= 1, decode_mode 0/1/2",
                      GPU_MAX_ROLLOUTS);
        return RT_EINVAL;
    }
    if (full) {
        if (!arena || !arena->base || cfg->num_kv_heads == 0 || cfg->num_q_heads == 0 ||
            cfg->num_q_heads % cfg->num_kv_heads || cfg->vocab == 0 || cfg->vocab > 32768u ||
            cfg->max_context < 16u || cfg->max_new_tokens == 0) {
            rt::set_error("rollout: full decode needs an arena, heads (q multiple of kv), "
                          "vocab 1..32768, max_context >= 16, max_new_tokens >= 1");
            return RT_EINVAL;
        }
        if (arena->block_size != rt_page_bytes(cfg->num_kv_heads)) {
            rt::set_error("rollout: arena block_size %zu != page size %llu", arena->block_size,
                          (unsigned long long)rt_page_bytes(cfg->num_kv_heads));
            return RT_EINVAL;
        }
    }
    rt_rollout *e = new (std::nothrow) rt_rollout();
    if (!e) {
        rt::set_error("rollout: out of host memory");
        return RT_ENOMEM;
    }
    e->cfg = *cfg;
    e->arena = arena;
    cudaGetDevice(&e->device);
    Dev &d = e->d;
    d.max_slots = cfg->max_slots;
    d.max_admit = cfg->max_admit;
    d.drop = cfg->drop_when_full ? 1u : 0u;
    d.decode = cfg->decode_mode;
    d.reward_mode = cfg->reward_mode;
    d.reward_seed = cfg->reward_seed;
    d.vocab = cfg->vocab;
    d.hq = cfg->num_q_heads;
    d.hkv = cfg->num_kv_heads;
    d.max_new = cfg->max_new_tokens;
    d.max_prefixes = cfg->max_prefixes;
    d.maxp = full ? (cfg->max_context + 15u) / 16u : 1u;
    d.ppriv = full ? (cfg->max_new_tokens + 16u + 15u) / 16u : 1u;
    d.max_passes = cfg->max_passes ? cfg->max_passes : (1ull << 40);
    d.idle_ns = (uint64_t)(cfg->idle_timeout_ms ? cfg->idle_timeout_ms : 10000u) * 1000000ull;
    d.logit_std = cfg->logit_std;

    cudaError_t err = cudaSuccess;
    auto ok = [&](cudaError_t x) { if (err == cudaSuccess) err = x; };
    const uint32_t S = d.max_slots;
    ok(dalloc(&d.io, 1));
    ok(dalloc(&d.ctl, 1));
    ok(dalloc(&d.ext, S));
    ok(dalloc(&d.seq_lens, S));
    ok(dalloc(&d.enable, S));
    ok(dalloc(&d.srows, S));
    ok(dalloc(&d.tokens, S));
    ok(cudaMallocHost(reinterpret_cast<void **>(&e->io_stage), sizeof(RtIo)));
    if (full) {
        ok(dalloc(&d.page_table, (size_t)S * d.maxp));
        ok(dalloc(&d.priv, (size_t)S * d.ppriv));
        ok(dalloc(&d.q, (size_t)S * d.hq * 128u));
        ok(dalloc(&d.attn_out, (size_t)S * d.hq * 128u));
        ok(dalloc(&d.logits, (size_t)S * d.vocab));
        d.cstride = rt_chunk_max_stride(d.vocab);
        ok(dalloc(&d.cmax, (size_t)S * d.cstride));
        const uint32_t npf = cfg->max_prefixes ? cfg->max_prefixes : 1u;
        ok(dalloc(&d.pf_len, npf));
        ok(dalloc(&d.pf_np, npf));
        ok(dalloc(&d.pf_off, npf));
        ok(dalloc(&d.pf_pages, cfg->max_prefix_pages ? cfg->max_prefix_pages : 1u));
        if (cfg->prefix_attention == RT_PREFIX_ATTN_GROUPED) {
            d.max_groups = (S + 1u) / 2u;  // groups have at least two members
            ok(dalloc(&d.groups, d.max_groups));
            ok(dalloc(&d.n_groups, 1));
            ok(dalloc(&d.skip, S));
        }
        ok(dalloc(&d.attn_chunks, 2u + S));
    }
    if (err != cudaSuccess) {
        engine_free(e);
        return rt::cuda_fail(err, "rollout: device allocation");
    }
    ok(cudaMemset(d.ctl, 0, sizeof(RtCtl)));  // counters read before a first launch are zero
    if (full) {
        e->pf_len_h = new (std::nothrow) uint32_t[npf_h(cfg)]();
        e->pf_off_h = new (std::nothrow) uint32_t[npf_h(cfg)]();
        if (!e->pf_len_h || !e->pf_off_h) {
            engine_free(e);
            rt::set_error("rollout: out of host memory");
            return RT_ENOMEM;
        }
        ok(cudaMemset(d.pf_len, 0, sizeof(uint32_t) * (cfg->max_prefixes ? cfg->max_prefixes : 1u)));
        ok(cudaMemset(d.pf_np, 0, sizeof(uint32_t) * (cfg->max_prefixes ? cfg->max_prefixes : 1u)));
        d.arena = reinterpret_cast<__nv_bfloat16 *>(arena->base);
        // reserve the private pages from the arena (lowest free blocks first)
        e->n_priv = S * d.ppriv;
        e->priv_blocks = static_cast<int64_t *>(malloc(sizeof(int64_t) * e->n_priv));
        int32_t *h = static_cast<int32_t *>(malloc(sizeof(int32_t) * e->n_priv));
        uint32_t got = 0;
        for (; got < e->n_priv; got++) {
            const int64_t b = arena_acquire(arena);
            if (b < 0 || b > INT32_MAX)
                break;
            e->priv_blocks[got] = b;
            h[got] = (int32_t)b;
        }
        if (got < e->n_priv) {
            e->n_priv = got;
            free(h);
            engine_free(e);
            rt::set_error("rollout: arena has fewer than %u free pages", S * d.ppriv);
            return RT_ENOMEM;
        }
        ok(cudaMemcpy(d.priv, h, sizeof(int32_t) * e->n_priv, cudaMemcpyHostToDevice));
        free(h);
        const uint64_t arena_pages = arena->capacity / arena->block_size;
        e->ap.num_seqs = S;
        e->ap.num_q_heads = d.hq;
        e->ap.num_kv_heads = d.hkv;
        e->ap.head_dim = 128u;
        e->ap.max_pages_per_seq = d.maxp;
        e->ap.max_seq_len = d.maxp * 16u;
        e->ap.arena_pages = arena_pages;
        e->ap.scale = 0.08838834764831845f;  // 1/sqrt(128)
        // Auto: with contexts beyond 64 pages, 16-page items.  A slot whose
        // GRPO group has no other active member attends its whole context
        // alone, and short items keep such slots off the pass's tail; the
        // schedule kernel's item table means the extra chunks of the other
        // slots cost nothing (configuration 4: 1.33 against 1.26 M tokens/s
        // with the plan's 48-page items).  Shorter contexts take the plan's
        // own rule.
        e->ap.chunk_pages = cfg->chunk_pages ? cfg->chunk_pages : (d.maxp > 64u ? 16u : 0u);
        e->ap.kv_evict_first = 0u;  // group members re-read shared prefix pages
        e->gp.max_groups = d.max_groups;
        e->gp.max_shared_pages = d.maxp;
        e->gp.chunk_pages = 0u;
        e->gp.reserved = 0u;
        e->attn_ws_bytes = d.max_groups ? rt_attn_grouped_workspace_bytes(&e->ap, &e->gp)
                                        : rt_attn_workspace_bytes(&e->ap);
        if (e->attn_ws_bytes == 0 ||
            rt::attn_item_shape(&e->ap, d.max_groups ? &e->gp : nullptr, &d.attn_cp, &d.attn_gcp,
                                &d.attn_mg) != RT_OK) {
            engine_free(e);
            return RT_EINVAL;
        }
        ok(cudaMalloc(&e->attn_ws, e->attn_ws_bytes));
        ok(cudaMemset(e->attn_ws, 0, e->attn_ws_bytes));
        if (err == cudaSuccess) {
            int rc = rt::attn_prepare(&e->ap);
            if (rc != RT_OK) {
                engine_free(e);
                return rc;
            }
        }
    }
    ok(cudaStreamCreateWithFlags(&e->cap, cudaStreamNonBlocking));
    if (err != cudaSuccess) {
        engine_free(e);
        return rt::cuda_fail(err, "rollout: setup");
    }
    // a model-decode engine builds its graph once its weights are attached
    if (cfg->decode_mode != RT_ROLLOUT_DECODE_MODEL) {
        int rc = engine_build_graph(e);
        if (rc != RT_OK) {
            engine_free(e);
            return rc;
        }
    }
    *out = e;
    return RT_OK;
}

extern "C" int rt_rollout_set_model(rt_rollout_t *e, const rt_model_weights_t *w)
{
    if (!e || !w || e->cfg.decode_mode != RT_ROLLOUT_DECODE_MODEL || !w->embed || !w->w_qkv ||
        !w->w_lm) {
        rt::set_error("rollout_set_model: needs a model-decode engine and three weight matrices");
        return RT_EINVAL;
    }
    Dev &d = e->d;
    if (w->d_model != d.hq * 128u || ((uintptr_t)w->embed | (uintptr_t)w->w_qkv |
                                       (uintptr_t)w->w_lm) % 16u) {
        rt::set_error("rollout_set_model: d_model must be num_q_heads * 128 (%u), weights "
                      "16-byte aligned", d.hq * 128u);
        return RT_EINVAL;
    }
    cudaError_t err = cudaDeviceSynchronize();  // no launch of this engine in flight
    if (err != cudaSuccess)
        return rt::cuda_fail(err, "rollout_set_model: sync");
    const uint32_t S = d.max_slots;
    d.dm = w->d_model;
    d.qkv_n = (d.hq + 2u * d.hkv) * 128u;
    if (!d.hin) {
        auto ok = [&](cudaError_t x) { if (err == cudaSuccess) err = x; };
        ok(dalloc(&d.hin, (size_t)S * d.dm));
        ok(dalloc(&d.hout, (size_t)S * d.dm));
        ok(dalloc(&d.qkv, (size_t)S * d.qkv_n));
        ok(dalloc(&d.emb_tok, S));
        ok(dalloc(&d.gemm_err, 1));
        ok(cudaMemset(d.hin, 0, sizeof(__nv_bfloat16) * S * d.dm));
        ok(cudaMemset(d.hout, 0, sizeof(__nv_bfloat16) * S * d.dm));
        ok(cudaMemset(d.gemm_err, 0, sizeof(int32_t)));
        if (err != cudaSuccess)
            return rt::cuda_fail(err, "rollout_set_model: buffers");
    }
    // K-splits of the LM head that fill the GPU, and their partial-sum workspace
    d.split_lm = gemm_splits(S, d.vocab, d.dm);
    rt_gemm_params_t gl = {S, d.vocab, d.dm, d.dm, d.dm, d.vocab, d.split_lm, 0u};
    const uint64_t need = rt_gemm_workspace_bytes(&gl);
    if (need > d.gemm_ws_bytes) {
        if (d.gemm_ws)
            cudaFree(d.gemm_ws);
        d.gemm_ws = nullptr;
        d.gemm_ws_bytes = 0;
        if ((err = cudaMalloc(&d.gemm_ws, need)) != cudaSuccess)
            return rt::cuda_fail(err, "rollout_set_model: projection workspace");
        d.gemm_ws_bytes = need;
    }
    if (!e->pre_x) {
        auto ok = [&](cudaError_t x) { if (err == cudaSuccess) err = x; };
        ok(dalloc(&e->pre_x, (size_t)kPrefillChunk * d.dm));
        ok(dalloc(&e->pre_kv, (size_t)kPrefillChunk * d.hkv * 256u));
        if (err != cudaSuccess)
            return rt::cuda_fail(err, "rollout_set_model: prefill scratch");
    }
    d.w_embed = static_cast<const __nv_bfloat16 *>(w->embed);
    d.w_qkv = static_cast<const __nv_bfloat16 *>(w->w_qkv);
    d.w_lm = static_cast<const __nv_bfloat16 *>(w->w_lm);
    if (!e->blas) {
        // cuBLAS handle and workspace for the QKV projection, and one call
        // outside capture (its first call loads its kernels)
        constexpr size_t kBlasWs = 32u << 20;
        if (cublasCreate(&e->blas) != CUBLAS_STATUS_SUCCESS) {
            e->blas = nullptr;
            rt::set_error("rollout_set_model: cublasCreate failed");
            return RT_ECUDA;
        }
        if ((err = cudaMalloc(&e->blas_ws, kBlasWs)) != cudaSuccess)
            return rt::cuda_fail(err, "rollout_set_model: cuBLAS workspace");
        if (cublasSetWorkspace(e->blas, e->blas_ws, kBlasWs) != CUBLAS_STATUS_SUCCESS) {
            rt::set_error("rollout_set_model: cublasSetWorkspace failed");
            return RT_ECUDA;
        }
    }
    {
        const int qrc = qkv_projection(e, e->cap);
        if (qrc != RT_OK)
            return qrc;
        if ((err = cudaStreamSynchronize(e->cap)) != cudaSuccess)
            return rt::cuda_fail(err, "rollout_set_model: QKV projection");
    }
    // kernel attributes before capture (the graph bakes the weight pointers in)
    int rc = rt::gemm_prepare();
    if (rc != RT_OK)
        return rc;
    if (e->exec) {
        cudaGraphExecDestroy(e->exec);
        e->exec = nullptr;
    }
    if (e->graph) {
        cudaGraphDestroy(e->graph);
        e->graph = nullptr;
    }
    return engine_build_graph(e);
}

extern "C" int rt_rollout_destroy(rt_rollout_t *e)
{
    if (e) {
        cudaDeviceSynchronize();
        engine_free(e);
    }
    return RT_OK;
}

extern "C" int rt_rollout_set_prefix(rt_rollout_t *e, uint32_t prefix_id, const int32_t *pages,
                                     uint32_t n_pages, uint32_t token_len)
{
    if (!e || (!pages && n_pages) || e->cfg.decode_mode == RT_ROLLOUT_DECODE_NONE) {
        rt::set_error("rollout_set_prefix: needs a full-decode engine and a page list");
        return RT_EINVAL;
    }
    if (prefix_id >= e->cfg.max_prefixes || (token_len + 15u) / 16u > n_pages ||
        token_len > e->d.maxp * 16u) {
        rt::set_error("rollout_set_prefix: prefix %u (max %u) with %u tokens needs %u pages (got %u) "
                      "and at most %u tokens (the context)",
                      prefix_id, e->cfg.max_prefixes, token_len, (token_len + 15u) / 16u, n_pages,
                      e->d.maxp * 16u);
        return RT_EINVAL;
    }
    if (e->pf_used + n_pages > e->cfg.max_prefix_pages) {
        rt::set_error("rollout_set_prefix: prefix page pool full (%u of %u)", e->pf_used,
                      e->cfg.max_prefix_pages);
        return RT_ENOMEM;
    }
    const uint64_t arena_pages = e->arena->capacity / e->arena->block_size;
    for (uint32_t i = 0; i < n_pages; i++)
        if (pages[i] < 0 || (uint64_t)pages[i] >= arena_pages) {
            rt::set_error("rollout_set_prefix: page %d outside the arena", pages[i]);
            return RT_EINVAL;
        }
    cudaError_t err = cudaMemcpy(e->d.pf_pages + e->pf_used, pages, sizeof(int32_t) * n_pages,
                                 cudaMemcpyHostToDevice);
    const uint32_t off = e->pf_used;
    if (err == cudaSuccess)
        err = cudaMemcpy(e->d.pf_len + prefix_id, &token_len, 4, cudaMemcpyHostToDevice);
    if (err == cudaSuccess)
        err = cudaMemcpy(e->d.pf_np + prefix_id, &n_pages, 4, cudaMemcpyHostToDevice);
    if (err == cudaSuccess)
        err = cudaMemcpy(e->d.pf_off + prefix_id, &off, 4, cudaMemcpyHostToDevice);
    if (err != cudaSuccess)
        return rt::cuda_fail(err, "rollout_set_prefix: copy");
    e->pf_len_h[prefix_id] = token_len;
    e->pf_off_h[prefix_id] = off;
    e->pf_used += n_pages;
    return RT_OK;
}

static int rollout_setup(rt_rollout_t *e, const rt_rollout_io_t *io, cudaStream_t s);

extern "C" int rt_rollout_prefill(rt_rollout_t *e, uint32_t prefix_id, const uint32_t *tokens,
                                  uint32_t n_tokens, void *stream)
{
    if (!e || e->cfg.decode_mode != RT_ROLLOUT_DECODE_MODEL || !e->d.w_embed) {
        rt::set_error("rollout_prefill: needs a model-decode engine with its weights attached");
        return RT_EINVAL;
    }
    if (prefix_id >= e->cfg.max_prefixes || e->pf_len_h[prefix_id] != n_tokens ||
        (n_tokens && !tokens)) {
        rt::set_error("rollout_prefill: prefix %u must be registered with exactly %u tokens",
                      prefix_id, n_tokens);
        return RT_EINVAL;
    }
    const Dev &d = e->d;
    cudaStream_t s = (cudaStream_t)stream;
    const int32_t *pages = d.pf_pages + e->pf_off_h[prefix_id];
    const uint32_t nkv = d.hkv * 256u;  // k then v rows of every kv head
    for (uint32_t c0 = 0; c0 < n_tokens; c0 += kPrefillChunk) {
        const uint32_t m = std::min(kPrefillChunk, n_tokens - c0);
        prefill_embed_kernel<<<m, 256, 0, s>>>(tokens + c0, d.w_embed, e->pre_x, d.dm, d.vocab,
                                               d.gemm_err);
        cudaError_t err = cudaGetLastError();
        if (err != cudaSuccess)
            return rt::cuda_fail(err, "rollout_prefill: embed launch");
        // the K / V rows of the QKV weight follow its hq * 128 q rows
        rt_gemm_params_t gp = {m, nkv, d.dm, d.dm, d.dm, nkv, gemm_splits(m, nkv, d.dm), 0u};
        while (gp.split_k > 1u && rt_gemm_workspace_bytes(&gp) > d.gemm_ws_bytes)
            gp.split_k--;  // K-splits only as far as the engine's workspace holds them
        int rc = rt_gemm_bf16(&gp, e->pre_x, d.w_qkv + (size_t)d.hq * 128u * d.dm, e->pre_kv,
                              d.gemm_ws, d.gemm_ws_bytes, d.gemm_err, s);
        if (rc != RT_OK)
            return rc;
        prefill_scatter_kernel<<<m, 256, 0, s>>>(e->pre_kv, pages, c0, d.hkv, d.arena);
        err = cudaGetLastError();
        if (err != cudaSuccess)
            return rt::cuda_fail(err, "rollout_prefill: scatter launch");
    }
    return RT_OK;
}

extern "C" size_t rt_trace_bytes(uint32_t capacity)
{
    if (capacity == 0 || (capacity & (capacity - 1u))) {
        rt::set_error("trace: capacity %u must be a power of two", capacity);
        return 0;
    }
    return offsetof(TraceRing, entries) + (size_t)capacity * sizeof(rt_trace_entry_t);
}

extern "C" int rt_trace_init(void *trace, uint32_t capacity, void *stream)
{
    if (!trace || rt_trace_bytes(capacity) == 0) {
        rt::set_error("trace_init: needs a buffer of rt_trace_bytes(capacity)");
        return RT_EINVAL;
    }
    TraceRing hdr;
    memset(&hdr, 0, offsetof(TraceRing, entries));
    hdr.capacity = capacity;
    cudaError_t err = cudaMemcpyAsync(trace, &hdr, offsetof(TraceRing, entries),
                                      cudaMemcpyHostToDevice, (cudaStream_t)stream);
    if (err == cudaSuccess)
        err = cudaStreamSynchronize((cudaStream_t)stream);
    return err == cudaSuccess ? RT_OK : rt::cuda_fail(err, "trace_init");
}

extern "C" int rt_trace_read(const void *trace, rt_trace_entry_t *out, uint32_t max,
                             uint64_t *appended, void *stream)
{
    if (!trace || (max && !out)) {
        rt::set_error("trace_read: null argument");
        return RT_EINVAL;
    }
    cudaStream_t s = (cudaStream_t)stream;
    TraceRing hdr;
    cudaError_t err = cudaMemcpyAsync(&hdr, trace, offsetof(TraceRing, entries),
                                      cudaMemcpyDeviceToHost, s);
    if (err == cudaSuccess)
        err = cudaStreamSynchronize(s);
    if (err != cudaSuccess)
        return rt::cuda_fail(err, "trace_read: header");
    if (appended)
        *appended = hdr.head;
    if (hdr.capacity == 0 || (hdr.capacity & (hdr.capacity - 1u))) {
        rt::set_error("trace_read: the buffer was not initialised with rt_trace_init");
        return RT_EINVAL;
    }
    const uint64_t avail = std::min<uint64_t>(hdr.head, hdr.capacity);
    const uint64_t n = std::min<uint64_t>(avail, max);
    const rt_trace_entry_t *ent =
        reinterpret_cast<const rt_trace_entry_t *>(static_cast<const uint8_t *>(trace) +
                                                   offsetof(TraceRing, entries));
    // the newest n records in append order: start at head - n (mod capacity)
    const uint64_t first = hdr.head - n;
    const uint64_t i0 = first & (hdr.capacity - 1u);
    const uint64_t run = std::min<uint64_t>(n, hdr.capacity - i0);
    if (run)
        err = cudaMemcpyAsync(out, ent + i0, run * sizeof(rt_trace_entry_t), cudaMemcpyDeviceToHost, s);
    if (err == cudaSuccess && n > run)
        err = cudaMemcpyAsync(out + run, ent, (n - run) * sizeof(rt_trace_entry_t),
                              cudaMemcpyDeviceToHost, s);
    if (err == cudaSuccess)
        err = cudaStreamSynchronize(s);
    return err == cudaSuccess ? RT_OK : rt::cuda_fail(err, "trace_read: records");
}

extern "C" int rt_rollout_set_trace(rt_rollout_t *e, void *trace)
{
    if (!e) {
        rt::set_error("rollout_set_trace: null engine");
        return RT_EINVAL;
    }
    cudaError_t err = cudaDeviceSynchronize();  // no launch of this engine in flight
    if (err != cudaSuccess)
        return rt::cuda_fail(err, "rollout_set_trace: sync");
    e->d.trace = static_cast<TraceRing *>(trace);
    if (!e->exec)
        return RT_OK;  // a model-decode engine captures its graph at rt_rollout_set_model
    cudaGraphExecDestroy(e->exec);
    e->exec = nullptr;
    cudaGraphDestroy(e->graph);
    e->graph = nullptr;
    return engine_build_graph(e);
}

extern "C" int rt_rollout_launch(rt_rollout_t *e, const rt_rollout_io_t *io, void *stream)
{
    if (e && !e->exec) {
        rt::set_error("rollout_launch: a model-decode engine needs rt_rollout_set_model first");
        return RT_EINVAL;
    }
    cudaStream_t s = (cudaStream_t)stream;
    int rc = rollout_setup(e, io, s);
    if (rc != RT_OK)
        return rc;
    cudaError_t err = cudaGraphLaunch(e->exec, s);
    if (err != cudaSuccess)
        return rt::cuda_fail(err, "rollout_launch");
    return RT_OK;
}

static int rollout_setup(rt_rollout_t *e, const rt_rollout_io_t *io, cudaStream_t s)
{
    if (!e || !io || !io->state || (!io->ring && !io->requests && io->n_requests)) {
        rt::set_error("rollout_launch: needs an engine, a state table and a request source");
        return RT_EINVAL;
    }
    if (io->ring && io->requests) {
        rt::set_error("rollout_launch: give either a request ring or a request array");
        return RT_EINVAL;
    }
    if (io->arrivals && (io->ring || io->arrival_unit > RT_ARRIVAL_NS)) {
        rt::set_error("rollout_launch: arrivals gate an array source only, in passes or ns");
        return RT_EINVAL;
    }
    // Pageable staging: cudaMemcpyAsync copies it before returning, so a
    // later launch cannot overwrite the block of an earlier one in flight.
    RtIo stage;
    RtIo *x = &stage;
    x->ring = io->ring;
    x->reqs = io->requests;
    x->n_reqs = io->ring ? 0u : io->n_requests;
    x->done_ring = io->done_ring;
    x->dones = io->dones;
    x->state = io->state;
    x->step_count = reinterpret_cast<unsigned long long *>(io->step_count);
    x->traj = io->trajectories;
    x->rewards = io->rewards;
    x->n_rows = io->n_rows;
    x->arrival_unit = io->arrival_unit;
    x->arrivals = io->ring ? nullptr : io->arrivals;
    cudaError_t err = cudaMemcpyAsync(e->d.io, x, sizeof(RtIo), cudaMemcpyHostToDevice, s);
    if (err == cudaSuccess)
        err = cudaMemsetAsync(e->d.ctl, 0, sizeof(RtCtl), s);
    if (err == cudaSuccess)
        err = cudaMemsetAsync(e->d.ext, 0, sizeof(SlotExt) * e->d.max_slots, s);
    if (err == cudaSuccess)
        err = cudaMemsetAsync(e->d.enable, 0, sizeof(uint32_t) * e->d.max_slots, s);
    if (err == cudaSuccess)
        err = cudaMemsetAsync(io->state, 0, sizeof(GpuRolloutState), s);
    if (err != cudaSuccess)
        return rt::cuda_fail(err, "rollout_launch: setup");
    return RT_OK;
}

// Host-stepped replay of the loop with CUDA events around every kernel of
// every pass (per-kernel durations for roofline reporting).  Same kernels,
// same data as rt_rollout_launch; the host synchronises once per pass.
extern "C" int rt_rollout_profile(rt_rollout_t *e, const rt_rollout_io_t *io, void *stream,
                                  rt_rollout_profile_t *out)
{
    return rt_rollout_profile_hook(e, io, stream, out, nullptr, nullptr);
}

extern "C" int rt_rollout_buffers(rt_rollout_t *e, rt_rollout_buffers_t *out)
{
    if (!e || !out || e->cfg.decode_mode == RT_ROLLOUT_DECODE_NONE) {
        rt::set_error("rollout_buffers: needs a full-decode engine and an output struct");
        return RT_EINVAL;
    }
    out->q = e->d.q;
    out->attn_out = e->d.attn_out;
    out->page_table = e->d.page_table;
    out->seq_lens = e->d.seq_lens;
    out->groups = e->d.groups;
    out->n_groups = e->d.n_groups;
    out->skip_pages = e->d.skip;
    out->max_pages = e->d.maxp;
    out->max_groups = e->d.max_groups;
    out->logits = e->d.logits;
    out->tokens = e->d.tokens;
    out->enable = e->d.enable;
    out->sample_rows = e->d.srows;
    out->hidden_in = e->d.hin;
    out->qkv = e->d.qkv;
    out->hidden_out = e->d.hout;
    out->embed_tokens = e->d.emb_tok;
    return RT_OK;
}

extern "C" int rt_rollout_profile_hook(rt_rollout_t *e, const rt_rollout_io_t *io, void *stream,
                                       rt_rollout_profile_t *out, rt_rollout_pass_hook_t hook,
                                       void *user)
{
    if (!e || !out || e->cfg.decode_mode == RT_ROLLOUT_DECODE_NONE) {
        rt::set_error("rollout_profile: needs a full-decode engine and an output struct");
        return RT_EINVAL;
    }
    if (!e->exec) {
        rt::set_error("rollout_profile: a model-decode engine needs rt_rollout_set_model first");
        return RT_EINVAL;
    }
    cudaStream_t s = (cudaStream_t)stream;
    int rc = rollout_setup(e, io, s);
    if (rc != RT_OK)
        return rc;
    memset(out, 0, sizeof(*out));
    cudaEvent_t ev[6];
    for (auto &x : ev)
        cudaEventCreate(&x);
    const uint32_t S = e->d.max_slots;
    int32_t *lens = new int32_t[S];
    SlotExt *ext = new SlotExt[S];
    const double tok_bytes = (double)e->d.hkv * 128.0 * 2.0 * 2.0;  // K+V bf16 per token
    cudaError_t err = cudaSuccess;
    for (uint64_t pass = 0; pass < e->d.max_passes; pass++) {
        cudaEventRecord(ev[5], s);
        schedule_kernel<<<1, kSched, 0, s>>>(e->d, 0, 0);
        rc = launch_decode(e, s, ev);
        if (rc != RT_OK)
            break;
        RtCtl c;
        err = cudaMemcpyAsync(lens, e->d.seq_lens, sizeof(int32_t) * S, cudaMemcpyDeviceToHost, s);
        if (err == cudaSuccess)
            err = cudaMemcpyAsync(ext, e->d.ext, sizeof(SlotExt) * S, cudaMemcpyDeviceToHost, s);
        if (err == cudaSuccess)
            err = cudaMemcpyAsync(&c, e->d.ctl, sizeof(c), cudaMemcpyDeviceToHost, s);
        if (err == cudaSuccess)
            err = cudaStreamSynchronize(s);
        if (err != cudaSuccess)
            break;
        float ms[5];
        cudaEventElapsedTime(&ms[0], ev[5], ev[0]);
        for (int k = 0; k < 4; k++)
            cudaEventElapsedTime(&ms[k + 1], ev[k], ev[k + 1]);
        out->ms_schedule += ms[0];
        out->ms_prepare += ms[1];
        out->ms_attention += ms[2];
        out->ms_logits += ms[3];
        out->ms_sample += ms[4];
        out->passes++;
        uint32_t active = 0;
        double uniq = 0.0;
        uint32_t seen[64];
        uint32_t n_seen = 0;
        for (uint32_t k = 0; k < S; k++) {
            if (lens[k] <= 0)
                continue;
            active++;
            out->attn_bytes_logical += (double)lens[k] * tok_bytes;
            const uint32_t pf = ext[k].prefix;
            uniq += (double)(lens[k] - (int32_t)ext[k].ctx_len) * tok_bytes;
            bool dup = false;
            for (uint32_t j = 0; j < n_seen; j++)
                dup |= seen[j] == pf;
            if (pf && !dup) {
                if (n_seen < 64)
                    seen[n_seen++] = pf;
                uniq += (double)ext[k].ctx_len * tok_bytes;
            } else if (!pf) {
                uniq += (double)ext[k].ctx_len * tok_bytes;
            }
        }
        out->attn_bytes_unique += uniq;
        out->sample_rows += active;
        out->attn_launches += active ? 1u : 0u;
        if (c.stop || c.error)
            break;
        if (hook && hook(user, pass) != 0)
            break;
    }
    for (auto &x : ev)
        cudaEventDestroy(x);
    delete[] lens;
    delete[] ext;
    if (err != cudaSuccess)
        return rt::cuda_fail(err, "rollout_profile");
    return rc;
}

extern "C" int rt_rollout_wait(rt_rollout_t *e, void *stream, rt_rollout_stats_t *st)
{
    if (!e) {
        rt::set_error("rollout_wait: null engine");
        return RT_EINVAL;
    }
    cudaStream_t s = (cudaStream_t)stream;
    RtCtl c;
    cudaError_t err = cudaStreamSynchronize(s);
    if (err == cudaSuccess)
        err = cudaMemcpy(&c, e->d.ctl, sizeof(c), cudaMemcpyDeviceToHost);
    if (err != cudaSuccess)
        return rt::cuda_fail(err, "rollout_wait");
    int32_t attn_err = 0, model_err = 0;
    if (e->attn_ws && rt_attn_workspace_error(e->attn_ws, stream, &attn_err) != RT_OK)
        return RT_ECUDA;
    if (e->d.gemm_err && (err = cudaMemcpy(&model_err, e->d.gemm_err, sizeof(int32_t),
                                           cudaMemcpyDeviceToHost)) != cudaSuccess)
        return rt::cuda_fail(err, "rollout_wait: model error word");
    if (st) {
        st->passes = c.passes;
        st->tokens = c.tokens;
        st->consumed = c.consumed;
        st->admitted = c.admitted;
        st->dropped = c.dropped;
        st->done = c.done;
        st->max_active = c.max_active;
        st->stopped_by_sentinel = c.sentinel;
        st->error = c.error;
        st->attn_error = attn_err;
        st->model_error = model_err;
        st->pad = 0;
    }
    if (c.error) {
        rt::set_error("rollout: loop stopped with error %d after %llu passes", c.error,
                      (unsigned long long)c.passes);
        return c.error;
    }
    if (attn_err) {
        rt::set_error("rollout: attention reported device error %d", attn_err);
        return RT_EDEVICE;
    }
    if (model_err) {
        rt::set_error("rollout: a projection kernel reported device error %d", model_err);
        return RT_EDEVICE;
    }
    return RT_OK;
}

extern "C" int rt_logits_synth(float *out, uint32_t vocab, uint64_t seed, uint32_t request_lo,
                               uint64_t token_index, float logit_std, void *stream)
{
    if (!out || vocab == 0) {
        rt::set_error("logits_synth: bad argument");
        return RT_EINVAL;
    }
    const uint32_t groups = (vocab + 3u) / 4u;
    logits_synth_kernel<<<(groups + 255u) / 256u, 256, 0, (cudaStream_t)stream>>>(
        out, vocab, seed, request_lo, token_index, logit_std);
    cudaError_t err = cudaGetLastError();
    return err == cudaSuccess ? RT_OK : rt::cuda_fail(err, "logits_synth: launch");
}

// Drop-in for the reference's rollout_worker launch: a per-device control
// block (allocated on the first call) and a persistent single-CTA kernel.
static std::mutex g_worker_mu;
static RtIo *g_worker_io[64] = {};
static RtCtl *g_worker_ctl[64] = {};

extern "C" int rt_rollout_worker_stats(void *stream, rt_rollout_stats_t *st)
{
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64 || !g_worker_ctl[dev] || !st) {
        rt::set_error("rollout_worker_stats: no worker was launched on this device");
        return RT_EINVAL;
    }
    RtCtl c;
    cudaError_t err = cudaMemcpyAsync(&c, g_worker_ctl[dev], sizeof(c), cudaMemcpyDeviceToHost,
                                      (cudaStream_t)stream);
    if (err == cudaSuccess)
        err = cudaStreamSynchronize((cudaStream_t)stream);
    if (err != cudaSuccess)
        return rt::cuda_fail(err, "rollout_worker_stats");
    memset(st, 0, sizeof(*st));
    st->passes = c.passes;
    st->tokens = c.tokens;
    st->consumed = c.consumed;
    st->admitted = c.admitted;
    st->dropped = c.dropped;
    st->done = c.done;
    st->max_active = c.max_active;
    st->stopped_by_sentinel = c.sentinel;
    st->error = c.error;
    return RT_OK;
}

extern "C" int rt_launch_rollout_worker(RequestRing *req_ring, DoneRing *done_ring,
                                        GpuRolloutState *state, uint64_t *step_count,
                                        uint32_t idle_timeout_ms, void *stream)
{
    std::mutex &mu = g_worker_mu;
    RtIo **io_dev = g_worker_io;
    RtCtl **ctl_dev = g_worker_ctl;
    if (!req_ring || !done_ring || !state) {
        rt::set_error("rollout_worker: null ring or state");
        return RT_EINVAL;
    }
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) {
        rt::set_error("rollout_worker: device index %d out of range", dev);
        return RT_EINVAL;
    }
    cudaStream_t s = (cudaStream_t)stream;
    cudaError_t err = cudaSuccess;
    {
        std::lock_guard<std::mutex> lk(mu);
        if (!io_dev[dev]) {
            err = cudaMalloc(&io_dev[dev], sizeof(RtIo));
            if (err == cudaSuccess)
                err = cudaMalloc(&ctl_dev[dev], sizeof(RtCtl));
            if (err != cudaSuccess)
                return rt::cuda_fail(err, "rollout_worker: control block");
        }
    }
    RtIo x;
    memset(&x, 0, sizeof(x));
    x.ring = req_ring;
    x.done_ring = done_ring;
    x.state = state;
    x.step_count = reinterpret_cast<unsigned long long *>(step_count);
    Dev d;
    memset(&d, 0, sizeof(d));
    d.max_slots = GPU_MAX_ROLLOUTS;
    d.max_admit = 1u;
    d.drop = 1u;
    d.decode = RT_ROLLOUT_DECODE_NONE;
    d.reward_mode = RT_REWARD_MOCK;
    d.max_passes = 1ull << 62;
    d.idle_ns = (uint64_t)(idle_timeout_ms ? idle_timeout_ms : 10000u) * 1000000ull;
    d.io = io_dev[dev];
    d.ctl = ctl_dev[dev];
    err = cudaMemcpyAsync(d.io, &x, sizeof(x), cudaMemcpyHostToDevice, s);
    if (err == cudaSuccess)
        err = cudaMemsetAsync(d.ctl, 0, sizeof(RtCtl), s);
    if (err != cudaSuccess)
        return rt::cuda_fail(err, "rollout_worker: setup");
    persistent_worker_kernel<<<1, kSched, 0, s>>>(d);
    err = cudaGetLastError();
    return err == cudaSuccess ? RT_OK : rt::cuda_fail(err, "rollout_worker: launch");
}
