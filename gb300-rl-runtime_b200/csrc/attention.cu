// attention.cu - paged GQA decode attention for sm_100a.
//
// Generalises the reference's single-head, single-block decode step
// (reference cu/attention_decode.cu:60-204: q.K^T * 1/sqrt(128), online
// softmax over 16-token tiles, .V) to paged grouped-query attention over the
// KV arena, built for B200's memory system:
//
//  * Work unit: one WARP owns one item = (sequence b, KV head h, chunk of
//    `chunk_pages` 16-token pages).  Warps never synchronise with each other,
//    so a warp in its prologue (page ids, Q fragment, first TMA round trip)
//    overlaps the steady state of the other warps on the SM.  Items are
//    numbered head-fastest: the KV heads of one sequence chunk, whose
//    (page, head) blocks are adjacent in the arena, run side by side.
//  * Staging: per page the warp's elected lane issues four 2-D TMA tensor
//    loads (K and V, two 64-column halves each, 128-byte swizzle) into one
//    8 KiB stage of the warp's kStages-deep ring, completion tracked by a
//    shared-memory mbarrier with transaction bytes (no multicast).
//  * Math: per page, S^T = K.Q^T and O^T += V^T.P^T on m16n8k16 bf16 tensor
//    cores with the page's 16 tokens (or 16 head dimensions) as the M rows
//    and the KV group's G <= 8 query heads as the N = 8 columns: 8 mma for S
//    and 8 per P term for O.  Softmax runs in registers in the log2 domain
//    (column max over the 8 lanes of a head); P is split into two bf16 terms
//    so that P.V keeps ~16 mantissa bits; movmatrix turns the S^T
//    accumulator into the B operand of the second product.
//  * Shared prefixes: a separate group kernel reads a GRPO group's common
//    prefix pages once and multiplies them against all members' queries
//    (16 query rows = 16/G sequences x G heads per tile); the sequence kernel
//    starts each grouped sequence from those partials.
//  * Split-K: the chunks of one (b, h) write unnormalised partials; the last
//    warp to arrive (per-(b,h) counter) merges them with the log-sum-exp rule
//    and resets the counter, so no second kernel launch is needed.
//
// HBM roofline: the kernel must move sum_b L_b * Hkv * 128 * 2 * 2 bytes of
// KV plus q/out; at ~4 flop/byte it sits far below the tensor ridge.
#include <cmath>
#include <cstdint>
#include <mutex>

#include "kv_layout.h"
#include "rlrt.h"
#include "rt_common.cuh"
#include "rt_internal.h"

namespace {

#ifndef RT_ATTN_STAGES
#define RT_ATTN_STAGES 2
#endif
#ifndef RT_ATTN_CTAS_PER_SM
#define RT_ATTN_CTAS_PER_SM 3
#endif
constexpr int kWarps = 4;            // warps (independent items) per CTA
constexpr int kStages = RT_ATTN_STAGES;          // pipeline depth per warp
constexpr int kCtasPerSm = RT_ATTN_CTAS_PER_SM;  // resident CTAs per SM (shared memory)
constexpr int kStageBytes = 8192;    // K (2 x 2 KiB halves) + V (2 x 2 KiB)
constexpr int kMaxChunkPages = 64;   // page ids live in two registers per lane
constexpr int kSmemBytes = kWarps * kStages * kStageBytes + 1024;  // + 1 KiB alignment slack
// The sequence kernel adds each warp's G query rows, kQRowWords words a row
// (64 + 4 padding, so that the fragment reads of 8 rows hit 8 banks).
constexpr int kQRowWords = 68;
template <int G>
constexpr int seq_smem_bytes()
{
    return kSmemBytes + kWarps * G * kQRowWords * 4;
}
constexpr uint64_t kWaitLimitNs = 2000000000ull;                    // 2 s per pipeline wait

enum : int32_t { kErrSeqLen = 1, kErrPage = 2, kErrTimeout = 3, kErrGroup = 4 };

struct AttnArgs {
    const __nv_bfloat16 *q;
    const int32_t *page_table;
    const int32_t *seq_lens;
    float *out;
    float *part_o;      // [B][Hkv][max_chunks][G][128]
    float *part_ml;     // [B][Hkv][max_chunks][G][2]  (max, sum) in log2 domain
    int32_t *counters;  // [B][Hkv]
    int32_t *error;
    uint32_t *n_counters;  // header word: counters used by this call
    unsigned long long *work_next;  // item dispenser (dynamic scheduling)
    unsigned int *work_done;        // warps that left the loop
    uint32_t num_seqs, num_q_heads, num_kv_heads, max_pages, max_chunks, chunk_pages, max_seq_len;
    uint64_t arena_pages;
    uint64_t n_items;
    float scale_log2;
    uint32_t evict_first;
    // shared-prefix groups (cascade); groups == nullptr disables them
    const rt_attn_group_t *groups;
    const uint32_t *n_groups;          // device count of valid group records
    const uint32_t *skip_pages;        // [B] pages covered by the sequence's group, or nullptr
    unsigned long long *group_next;    // CTA-level dispenser of group items
    unsigned int *group_done;          // CTAs that left the group phase
    uint32_t max_groups, gchunk_pages, max_gchunks;
    uint32_t slots;                    // partial slots per (b, h): max_gchunks + max_chunks
    const uint32_t *dyn_chunks;        // this launch's largest chunk count (device), or nullptr
};

// The shared-prefix (group) kernel uses the CTA's whole ring.  Alone it is
// faster with 2 CTAs per SM and 12 stages, but in the loop the sequence
// kernel (a programmatic dependent) overlaps it, and 3 CTAs per SM, whose
// idle CTAs exit at once and free their SMs, gave the shorter pass
// (attention 60.3 against 64.0 us per pass, same box).
#ifndef RT_ATTN_GROUP_STAGES
#define RT_ATTN_GROUP_STAGES (kWarps * kStages)
#endif
#ifndef RT_ATTN_GROUP_CTAS_PER_SM
#define RT_ATTN_GROUP_CTAS_PER_SM kCtasPerSm
#endif
constexpr int kGroupStages = RT_ATTN_GROUP_STAGES;  // the CTA's whole ring, shared by its warps
constexpr int kGroupCtasPerSm = RT_ATTN_GROUP_CTAS_PER_SM;
constexpr int kGroupSmemBytes = kGroupStages * kStageBytes + 1024;
constexpr uint32_t kMaxGroupMembers = 16;

__device__ __forceinline__ void flag_error(int32_t *err, int32_t code)
{
    atomicCAS(err, 0, code);
}

// Partial slots of (b, h): group-prefix chunks use slots [0, max_gchunks),
// the sequence's own chunks use [max_gchunks, max_gchunks + max_chunks).

// Log-sum-exp merge of all partials of (b, h) into out; called by one warp.
// Latency-bound (L2 round trips), so the loads are issued wide: first the
// (max, sum) pairs of all parts x rows across the lanes, reduced per row with
// shuffles (row = lane % G is kept by xor offsets >= G), then per row the
// partial outputs four parts at a time, each lane owning 4 of the 128 dims.
template <int G>
__device__ __forceinline__ void merge_parts(const AttnArgs &a, size_t bh, uint32_t b, uint32_t h,
                                            uint32_t n_g, uint32_t n_s)
{
    const int lane = threadIdx.x & 31;
    const uint32_t n = n_g + n_s, pairs = n * G;
    auto slot_of = [&](uint32_t k) { return k < n_g ? k : a.max_gchunks + (k - n_g); };
    auto ml_at = [&](uint32_t k, uint32_t row) {
        return __ldcg(reinterpret_cast<const float2 *>(
            &a.part_ml[((bh * a.slots + slot_of(k)) * G + row) * 2]));
    };
    float m_lane = -INFINITY;
    for (uint32_t j = lane; j < pairs; j += 32)
        m_lane = fmaxf(m_lane, ml_at(j / G, j % G).x);
#pragma unroll
    for (int off = 16; off >= G; off >>= 1)
        m_lane = fmaxf(m_lane, __shfl_xor_sync(0xffffffffu, m_lane, off));
    float l_lane = 0.0f;
    for (uint32_t j = lane; j < pairs; j += 32) {
        const float2 ml = ml_at(j / G, j % G);
        l_lane += ml.y * rt::fast_exp2(ml.x - m_lane);
    }
#pragma unroll
    for (int off = 16; off >= G; off >>= 1)
        l_lane += __shfl_xor_sync(0xffffffffu, l_lane, off);

#pragma unroll
    for (int row = 0; row < G; row++) {
        const float M = __shfl_sync(0xffffffffu, m_lane, row);
        const float inv = 1.0f / __shfl_sync(0xffffffffu, l_lane, row);
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        uint32_t k = 0;
        for (; k + 4u <= n; k += 4u) {
            float2 ml[4];
            float4 v[4];
#pragma unroll
            for (int u = 0; u < 4; u++) {
                const size_t pi = (bh * a.slots + slot_of(k + u)) * G + row;
                ml[u] = __ldcg(reinterpret_cast<const float2 *>(&a.part_ml[pi * 2]));
                v[u] = __ldcg(reinterpret_cast<const float4 *>(&a.part_o[pi * 128 + lane * 4]));
            }
#pragma unroll
            for (int u = 0; u < 4; u++) {
                const float wt = rt::fast_exp2(ml[u].x - M);
                acc.x += v[u].x * wt;
                acc.y += v[u].y * wt;
                acc.z += v[u].z * wt;
                acc.w += v[u].w * wt;
            }
        }
        for (; k < n; k++) {
            const size_t pi = (bh * a.slots + slot_of(k)) * G + row;
            const float wt = rt::fast_exp2(__ldcg(&a.part_ml[pi * 2]) - M);
            const float4 v = __ldcg(reinterpret_cast<const float4 *>(&a.part_o[pi * 128 + lane * 4]));
            acc.x += v.x * wt;
            acc.y += v.y * wt;
            acc.z += v.z * wt;
            acc.w += v.w * wt;
        }
        *reinterpret_cast<float4 *>(a.out + ((size_t)b * a.num_q_heads + (size_t)h * G + row) * 128 +
                                    lane * 4) =
            make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv);
    }
}

// Sequence items: one warp per item; see the file comment.
//
// The tile is transposed relative to the usual decode formulation, because
// a KV group has only G <= 8 query heads: S^T = K.Q^T takes the page's 16
// tokens as the M rows of m16n8k16 and the G heads as its N = 8 columns, and
// O^T = V^T.P^T takes 16 head dimensions as M and the heads as N.  That is 8
// mma for S and 8 per P term for O per page, half of what 16-row query tiles
// (12 of them zero for G = 4) cost.  The S^T accumulator becomes the B
// operand of the second product through one movmatrix transpose per 8x8 block.
// A sequence item as one warp sees it: which (sequence, KV head, chunk), its
// page range and page ids (lane i holds item pages i and 32 + i), and what
// is left to do.  Filled by seq_setup from the item number alone plus three
// small loads (length, group coverage, the page-table row).
struct SeqItem {
    uint32_t b, h, n_g;
    int chunk, L, n_chunks, p_begin, n_mine;
    int pg_lo, pg_hi;
    uint32_t kind;  // kSeqNone: nothing; kSeqZero: write a zero output; kSeqWork: pages or a group fold
};
enum : uint32_t { kSeqNone = 0, kSeqZero = 1, kSeqWork = 2 };

// The launch's items, long ones first and the short ones - chunk 0: the
// remainders, folds and zero outputs - last, which keeps the tail short.
// By default they are (chunk from the highest index down, sequence, KV head)
// up to the plan's chunk count (from max_seq_len); chunks past a sequence's
// end are empty items.  When the caller publishes this launch's items on the
// device (the rollout loop's schedule kernel does: dyn_chunks[0] = the
// largest chunk count, [1] = all full chunks, i.e. chunks >= 1, [2 + b] =
// the full chunks of the sequences before b), there are no empty items:
// with one chunk per sequence the count alone says so, otherwise each CTA
// copies the prefix table to shared memory and hands out every full chunk,
// sequence by sequence (a binary search finds its sequence), then chunk 0
// of every sequence.
constexpr uint32_t kPlanSeqs = 512;
struct SeqPlan {
    uint32_t max_chunks;
    uint64_t n_items;
    const uint32_t *pre;  // shared-memory prefix table, or nullptr
    uint64_t n_full;      // full chunks (units of num_kv_heads items) in table order
};
__device__ __forceinline__ SeqPlan seq_plan(const AttnArgs &a, uint32_t *s_pre)
{
    SeqPlan pl;
    pl.max_chunks = a.max_chunks;
    pl.pre = nullptr;
    pl.n_full = 0;
    if (a.dyn_chunks) {
        const uint32_t c = a.dyn_chunks[0];
        pl.max_chunks = c < 1u ? 1u : (c < a.max_chunks ? c : a.max_chunks);
        if (pl.max_chunks > 1u && a.num_seqs <= kPlanSeqs) {
            for (uint32_t b = threadIdx.x; b < a.num_seqs; b += blockDim.x)
                s_pre[b] = a.dyn_chunks[2u + b];
            pl.n_full = a.dyn_chunks[1];
            pl.pre = s_pre;
            __syncthreads();
            pl.n_items = (pl.n_full + a.num_seqs) * a.num_kv_heads;
            return pl;
        }
    }
    pl.n_items = (uint64_t)a.num_seqs * a.num_kv_heads * pl.max_chunks;
    return pl;
}

template <int G>
__device__ __forceinline__ SeqItem seq_setup(const AttnArgs &a, const SeqPlan &pl, uint64_t item)
{
    const int lane = threadIdx.x & 31;
    SeqItem it;
    it.kind = kSeqNone;
    it.n_mine = 0;
    it.n_g = 0;
    it.n_chunks = 0;
    it.p_begin = 0;
    it.pg_lo = it.pg_hi = 0;
    it.L = 0;
    it.b = it.h = 0;
    it.chunk = 1;
    if (item >= pl.n_items)
        return it;
    const uint32_t B = a.num_seqs, Hkv = a.num_kv_heads;
    it.h = (uint32_t)(item % Hkv);
    const uint64_t unit = item / Hkv;
    int from_top = -1;  // table order: a full chunk's rank below its sequence's top chunk
    if (pl.pre) {
        if (unit < pl.n_full) {
            uint32_t lo = 0, hi = B;  // the last b with pre[b] <= unit
            while (hi - lo > 1u) {
                const uint32_t mid = (lo + hi) >> 1;
                if ((uint64_t)pl.pre[mid] <= unit)
                    lo = mid;
                else
                    hi = mid;
            }
            it.b = lo;
            from_top = (int)(unit - pl.pre[lo]);
        } else {
            it.b = (uint32_t)(unit - pl.n_full);
            it.chunk = 0;
        }
    } else {
        it.b = (uint32_t)(unit % B);
        it.chunk = (int)pl.max_chunks - 1 - (int)(unit / B);
    }
    const int L = a.seq_lens[it.b];
    const uint32_t skip_raw = a.skip_pages ? a.skip_pages[it.b] : 0u;
    it.L = L;
    const rt::AttnSeqShape sh = rt::attn_seq_shape(L, skip_raw, a.max_seq_len, a.max_pages,
                                                   a.gchunk_pages, a.max_gchunks, a.chunk_pages);
    if (from_top >= 0) {
        it.chunk = sh.n_chunks - 1 - from_top;
        if (it.chunk < 1) {  // the table disagrees with the lengths
            if (lane == 0)
                flag_error(a.error, kErrSeqLen);
            return it;
        }
    }
    if (sh.bad_len) {
        if (lane == 0 && it.chunk == 0)
            flag_error(a.error, kErrSeqLen);
        return it;
    }
    if (L == 0) {
        if (it.chunk == 0)
            it.kind = kSeqZero;
        return it;
    }
    if (sh.bad_skip)
        flag_error(a.error, kErrGroup);
    // a published chunk count below this sequence's would drop its top chunks
    if (sh.n_chunks > (int)pl.max_chunks && it.chunk == 0 && lane == 0)
        flag_error(a.error, kErrSeqLen);
    const int cp = (int)a.chunk_pages;
    it.n_g = sh.n_g;
    it.n_chunks = sh.n_chunks;
    if (it.chunk < 0 || it.chunk >= it.n_chunks)
        return it;
    const int rem = (sh.n_pages - sh.skip) - (it.n_chunks - 1) * cp;  // pages of chunk 0 (may be 0)
    it.p_begin = sh.skip + (it.chunk == 0 ? 0 : rem + (it.chunk - 1) * cp);
    it.n_mine = it.chunk == 0 ? max(0, rem) : cp;
    it.kind = kSeqWork;
    const int32_t *ptab = a.page_table + (size_t)it.b * a.max_pages + it.p_begin;
    if (lane < it.n_mine)
        it.pg_lo = ptab[lane];
    if (lane + 32 < it.n_mine)
        it.pg_hi = ptab[lane + 32];
    const bool bad = (lane < it.n_mine && (it.pg_lo < 0 || (uint64_t)it.pg_lo >= a.arena_pages)) ||
                     (lane + 32 < it.n_mine && (it.pg_hi < 0 || (uint64_t)it.pg_hi >= a.arena_pages));
    if (bad) {
        flag_error(a.error, kErrPage);
        if (it.pg_lo < 0 || (uint64_t)it.pg_lo >= a.arena_pages)
            it.pg_lo = 0;
        if (it.pg_hi < 0 || (uint64_t)it.pg_hi >= a.arena_pages)
            it.pg_hi = 0;
    }
    return it;
}

// Page i of the item into ring slot `ctr` (the warp's ctr-th issued page):
// lane 0 issues the four 2-D TMA loads (K and V halves) on that stage's
// mbarrier.
__device__ __forceinline__ void seq_issue(const CUtensorMap &kv_map, const AttnArgs &a,
                                          const SeqItem &it, int i, uint32_t ctr, uint32_t stage0,
                                          uint64_t (&bars)[kStages], uint64_t policy)
{
    const int pg = __shfl_sync(0xffffffffu, i < 32 ? it.pg_lo : it.pg_hi, i & 31);
    if ((threadIdx.x & 31) == 0) {
        const uint32_t s = ctr % (uint32_t)kStages;
        const uint32_t bar = rt::smem_u32(&bars[s]);
        const uint32_t dst = stage0 + s * (uint32_t)kStageBytes;
        const int32_t row_k = (int32_t)(((int64_t)pg * a.num_kv_heads + it.h) * 32);
        rt::mbar_arrive_expect_tx(bar, (uint32_t)kStageBytes);
        rt::tma_load_2d(dst, &kv_map, 0, row_k, bar, policy);
        rt::tma_load_2d(dst + 2048u, &kv_map, 64, row_k, bar, policy);
        rt::tma_load_2d(dst + 4096u, &kv_map, 0, row_k + 16, bar, policy);
        rt::tma_load_2d(dst + 6144u, &kv_map, 64, row_k + 16, bar, policy);
    }
}

// The item's G query rows (bf16 pairs) into the warp's shared buffer: row r
// at qs + r * kQRowWords.  Plain loads: the warp waits for them while the
// pages already issued are in flight.
template <int G>
__device__ __forceinline__ void seq_copy_q(const AttnArgs &a, const SeqItem &it, uint32_t *qs)
{
    const int lane = threadIdx.x & 31;
    const uint32_t *src = reinterpret_cast<const uint32_t *>(
        a.q + ((size_t)it.b * a.num_q_heads + (size_t)it.h * G) * 128);
    uint32_t v[2 * G];
#pragma unroll
    for (int k = 0; k < 2 * G; k++)
        v[k] = src[k * 32 + lane];
#pragma unroll
    for (int k = 0; k < 2 * G; k++) {
        const int w = k * 32 + lane;  // word w of the G x 64-word block
        qs[(w >> 6) * kQRowWords + (w & 63)] = v[k];
    }
}

// The end of an item: the lane sums of the softmax denominators, the fold of
// the group's prefix partials (chunk 0 of a grouped sequence), then either
// the normalised output (one chunk) or this chunk's partial, merged by the
// last chunk to arrive.
template <int G>
__device__ __forceinline__ void seq_finalize(const AttnArgs &a, const SeqItem &it, float (&o)[8][4],
                                             float m0, float m1, float l0, float l1)
{
    const int lane = threadIdx.x & 31;
    const int r = lane >> 2, q4 = lane & 3;
    const int hd0 = 2 * q4, hd1 = 2 * q4 + 1;
    const uint32_t b = it.b, h = it.h, n_g = it.n_g, Hq = a.num_q_heads;
    const int chunk = it.chunk, n_chunks = it.n_chunks;
    const size_t bh = (size_t)b * a.num_kv_heads + h;
    if (it.kind == kSeqZero) {
        for (int i = lane; i < G * 128; i += 32)
            a.out[((size_t)b * Hq + (size_t)h * G) * 128 + i] = 0.0f;
        return;
    }
    if (it.kind != kSeqWork)
        return;
#pragma unroll
    for (int off = 4; off < 32; off <<= 1) {
        l0 += __shfl_xor_sync(0xffffffffu, l0, off);
        l1 += __shfl_xor_sync(0xffffffffu, l1, off);
    }

    if (chunk == 0 && n_g) {
        // Fold in the group's prefix partials.  They come from the group
        // kernel launched just before this one as a programmatic dependent
        // launch, so this is where its completion is awaited - after this
        // warp's own pages, by when it has usually finished.
        rt::grid_dep_wait();
        const size_t pi0 = (bh * a.slots) * G;
        float M0 = m0, M1 = m1;
        for (uint32_t k = 0; k < n_g; k++) {
            if (hd0 < G)
                M0 = fmaxf(M0, a.part_ml[(pi0 + (size_t)k * G + hd0) * 2]);
            if (hd1 < G)
                M1 = fmaxf(M1, a.part_ml[(pi0 + (size_t)k * G + hd1) * 2]);
        }
        // rescale this warp's suffix state (exp2(-inf) = 0 when it had no pages)
        const float c0 = hd0 < G ? rt::fast_exp2(m0 - M0) : 0.0f;
        const float c1 = hd1 < G ? rt::fast_exp2(m1 - M1) : 0.0f;
        l0 *= c0;
        l1 *= c1;
#pragma unroll
        for (int dd = 0; dd < 8; dd++) {
            o[dd][0] *= c0;
            o[dd][2] *= c0;
            o[dd][1] *= c1;
            o[dd][3] *= c1;
        }
        for (uint32_t k = 0; k < n_g; k++) {
            const size_t pa = pi0 + (size_t)k * G;
            float w0 = 0.0f, w1 = 0.0f;
            const float *s0 = a.part_o + (pa + (hd0 < G ? hd0 : 0)) * 128 + r;
            const float *s1 = a.part_o + (pa + (hd1 < G ? hd1 : 0)) * 128 + r;
            if (hd0 < G) {
                const float2 ml = *reinterpret_cast<const float2 *>(&a.part_ml[(pa + hd0) * 2]);
                w0 = rt::fast_exp2(ml.x - M0);
                l0 += ml.y * w0;
            }
            if (hd1 < G) {
                const float2 ml = *reinterpret_cast<const float2 *>(&a.part_ml[(pa + hd1) * 2]);
                w1 = rt::fast_exp2(ml.x - M1);
                l1 += ml.y * w1;
            }
#pragma unroll
            for (int dd = 0; dd < 8; dd++) {
                if (hd0 < G) {
                    o[dd][0] += s0[16 * dd] * w0;
                    o[dd][2] += s0[16 * dd + 8] * w0;
                }
                if (hd1 < G) {
                    o[dd][1] += s1[16 * dd] * w1;
                    o[dd][3] += s1[16 * dd + 8] * w1;
                }
            }
        }
        m0 = M0;
        m1 = M1;
    }

    if (n_chunks == 1) {
        const float i0 = 1.0f / l0, i1 = 1.0f / l1;
        float *d0 = a.out + ((size_t)b * Hq + (size_t)h * G + hd0) * 128 + r;
        float *d1 = a.out + ((size_t)b * Hq + (size_t)h * G + hd1) * 128 + r;
#pragma unroll
        for (int dd = 0; dd < 8; dd++) {
            if (hd0 < G) {
                d0[16 * dd] = o[dd][0] * i0;
                d0[16 * dd + 8] = o[dd][2] * i0;
            }
            if (hd1 < G) {
                d1[16 * dd] = o[dd][1] * i1;
                d1[16 * dd + 8] = o[dd][3] * i1;
            }
        }
        return;
    }

    // ---- split-K: write this chunk's partial; the last part to arrive merges ----
    {
        const size_t pi = (bh * a.slots + a.max_gchunks + chunk) * G;
        float *d0 = a.part_o + (pi + hd0) * 128 + r;
        float *d1 = a.part_o + (pi + hd1) * 128 + r;
#pragma unroll
        for (int dd = 0; dd < 8; dd++) {
            if (hd0 < G) {
                d0[16 * dd] = o[dd][0];
                d0[16 * dd + 8] = o[dd][2];
            }
            if (hd1 < G) {
                d1[16 * dd] = o[dd][1];
                d1[16 * dd + 8] = o[dd][3];
            }
        }
        if (r == 0) {
            if (hd0 < G)
                *reinterpret_cast<float2 *>(a.part_ml + (pi + hd0) * 2) = make_float2(m0, l0);
            if (hd1 < G)
                *reinterpret_cast<float2 *>(a.part_ml + (pi + hd1) * 2) = make_float2(m1, l1);
        }
    }
    __threadfence();
    __syncwarp();
    int prev = 0;
    if (lane == 0)
        prev = atomicAdd(&a.counters[bh], 1);
    prev = __shfl_sync(0xffffffffu, prev, 0);
    if (prev != n_chunks - 1)
        return;
    __threadfence();
    merge_parts<G>(a, bh, b, h, 0u, (uint32_t)n_chunks);
    if (lane == 0)
        a.counters[bh] = 0;
    return;
}

// A warp's items, one after another, with the next item prefetched.  Its
// number is claimed from the global dispenser when the current item starts
// (one item ahead, so warps hold no more work than they can start); its
// setup loads (length, group coverage, page ids) and query rows follow the
// current item's first page, so they wait behind the pages in flight, and
// its first pages go into ring stages as the current item frees them: an
// item's first page is usually resident when it starts.  Returns when the
// dispenser is empty or a pipeline wait expired (flagged).
template <int G>
__device__ __forceinline__ void run_seq_items(const CUtensorMap &kv_map, const AttnArgs &a,
                                              const SeqPlan &pl, uint32_t stage0,
                                              uint8_t *base_ptr, uint32_t base_u32,
                                              uint64_t (&bars)[kStages], uint64_t policy,
                                              uint32_t *qs)
{
    const int lane = threadIdx.x & 31;
    const int r = lane >> 2, q4 = lane & 3;
    const int hd0 = 2 * q4, hd1 = 2 * q4 + 1;
    // ldmatrix row addresses (swizzled 16-byte chunk = chunk ^ row%8): lane
    // l points at token 8*((l/8)>>1) + l%8 and the (l/8)&1 half of a 16-dim
    // block, so the four 8x8 matrices are (tokens lo|hi) x (dims lo|hi).
    const int mi = lane >> 3, rr = lane & 7;
    const uint32_t t_row = (uint32_t)((((mi >> 1) << 3) + rr) * 128);
    uint32_t phases = 0, issued = 0, used = 0;  // ring: per-stage parity, pages issued / consumed
    unsigned long long grab = 0;
    if (lane == 0)
        grab = atomicAdd(a.work_next, 1ull);
    uint64_t id = __shfl_sync(0xffffffffu, grab, 0);
    SeqItem cur = seq_setup<G>(a, pl, id);
    // An empty item (nothing to write) costs only its setup: when one is
    // found, the number of the item after it is claimed at once, so the
    // claim's round trip overlaps the work still ahead.  A real item is
    // still claimed only when its predecessor starts.
    bool claimed = false;
    if (cur.kind == kSeqNone && id < pl.n_items) {
        if (lane == 0)
            grab = atomicAdd(a.work_next, 1ull);
        claimed = true;
    }
    int cur_iss = 0;
    // (the ring is idle: order the mbarrier set-up before the first TMA writes)
    rt::fence_proxy_async_smem();
    for (; cur_iss < cur.n_mine && cur_iss < kStages; cur_iss++)
        seq_issue(kv_map, a, cur, cur_iss, issued++, stage0, bars, policy);
    if (cur.n_mine > 0)
        seq_copy_q<G>(a, cur, qs);
    __syncwarp();
    while (id < pl.n_items) {
        if (lane == 0 && !claimed)
            grab = atomicAdd(a.work_next, 1ull);  // the next item, in flight meanwhile
        claimed = false;
        // Q as the B operand (col-major 16 dims x 8 heads): lane holds head
        // r, dims 16j + 2q4 (+1) and 16j + 8 + 2q4 (+1); heads >= G are zero.
        uint32_t qb[8][2];
        {
            const uint32_t *qrow = qs + (r < G ? r : 0) * kQRowWords;
#pragma unroll
            for (int j = 0; j < 8; j++) {
                qb[j][0] = r < G ? qrow[8 * j + q4] : 0u;
                qb[j][1] = r < G ? qrow[8 * j + 4 + q4] : 0u;
            }
        }
        __syncwarp();
        uint64_t id_n = pl.n_items;
        SeqItem nxt{};
        bool have_nxt = false;
        int nxt_iss = 0;
        // the next item's setup and query rows (qs is free: this item's
        // fragment is in registers)
        auto setup_next = [&]() {
            id_n = __shfl_sync(0xffffffffu, grab, 0);
            nxt = seq_setup<G>(a, pl, id_n);
            if (nxt.n_mine > 0)
                seq_copy_q<G>(a, nxt, qs);
            if (nxt.kind == kSeqNone && id_n < pl.n_items) {
                if (lane == 0)
                    grab = atomicAdd(a.work_next, 1ull);
                claimed = true;
            }
            have_nxt = true;
        };
        // Online-softmax state: lane owns heads 2q4, 2q4 + 1 and dims 16dd + r,
        // 16dd + r + 8 of the O^T tiles.
        float o[8][4];
#pragma unroll
        for (int n = 0; n < 8; n++)
            o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.0f;
        float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.0f, l1 = 0.0f;
        for (int i = 0; i < cur.n_mine; i++) {
            const int s = (int)(used % (uint32_t)kStages);
            const bool ok = rt::mbar_wait_bounded(rt::smem_u32(&bars[s]), (phases >> s) & 1u,
                                                  kWaitLimitNs);
            if (!__all_sync(0xffffffffu, ok)) {
                if (lane == 0)
                    flag_error(a.error, kErrTimeout);
                // give the copies still in flight a bounded chance to land
                // before the shared memory is released
                for (uint32_t k = used; k < issued; k++) {
                    const uint32_t s2 = k % (uint32_t)kStages;
                    (void)rt::mbar_wait_bounded(rt::smem_u32(&bars[s2]), (phases >> s2) & 1u,
                                                kWaitLimitNs / 4);
                    phases ^= 1u << s2;
                }
                return;
            }
            phases ^= 1u << s;
            used++;
        const uint32_t st = stage0 + (uint32_t)(s * kStageBytes);
        const int valid = min(16, cur.L - (cur.p_begin + i) * 16);
        if (valid < 16) {
            // Tail page: zero the V rows past the sequence end so that
            // P = 0 never meets non-finite stale data.
            uint8_t *vbase = base_ptr + (st - base_u32) + 4096;
            for (int idx = lane; idx < (16 - valid) * 2 * 8; idx += 32) {
                const int row = valid + idx / 16, halfc = idx % 16;
                *reinterpret_cast<uint4 *>(vbase + (halfc >> 3) * 2048 + row * 128 +
                                           (halfc & 7) * 16) = make_uint4(0, 0, 0, 0);
            }
            __syncwarp();
        }

        // S^T = K Q^T: 16 tokens x 8 heads, two accumulators (even / odd
        // 16-dim steps) to halve the dependent mma chain.
        float se[4] = {0.f, 0.f, 0.f, 0.f}, so[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int j = 0; j < 8; j++) {
            const int c = ((j & 3) << 1) + (mi & 1);
            const uint32_t addr = st + (uint32_t)((j >> 2) * 2048) + t_row + (uint32_t)((c ^ rr) << 4);
            uint32_t k0, k1, k2, k3;
            rt::ldsm_x4(addr, k0, k1, k2, k3);
            const uint32_t ka[4] = {k0, k2, k1, k3};
            if (j & 1)
                rt::mma_bf16_16816(so, ka, qb[j][0], qb[j][1]);
            else
                rt::mma_bf16_16816(se, ka, qb[j][0], qb[j][1]);
        }
        // lane: tokens r (x0: head hd0, x1: head hd1) and r + 8 (x2, x3)
        float x0 = (se[0] + so[0]) * a.scale_log2, x1 = (se[1] + so[1]) * a.scale_log2;
        float x2 = (se[2] + so[2]) * a.scale_log2, x3 = (se[3] + so[3]) * a.scale_log2;
        if (valid < 16) {
            if (r >= valid) x0 = x1 = -INFINITY;
            if (r + 8 >= valid) x2 = x3 = -INFINITY;
        }
        // max over the 16 tokens of each head: the 8 lanes of a column
        float mx0 = fmaxf(x0, x2), mx1 = fmaxf(x1, x3);
#pragma unroll
        for (int off = 4; off < 32; off <<= 1) {
            mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, off));
            mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, off));
        }
        const float n0 = fmaxf(m0, mx0), n1 = fmaxf(m1, mx1);
        const float c0 = rt::fast_exp2(m0 - n0), c1 = rt::fast_exp2(m1 - n1);
        const float p0 = rt::fast_exp2(x0 - n0), p1 = rt::fast_exp2(x1 - n1);
        const float p2 = rt::fast_exp2(x2 - n0), p3 = rt::fast_exp2(x3 - n1);
        l0 = l0 * c0 + (p0 + p2);
        l1 = l1 * c1 + (p1 + p3);
        m0 = n0;
        m1 = n1;
#pragma unroll
        for (int dd = 0; dd < 8; dd++) {
            o[dd][0] *= c0;
            o[dd][2] *= c0;
            o[dd][1] *= c1;
            o[dd][3] *= c1;
        }
        // P^T as the B operand: transpose the two 8x8 (token x head) blocks;
        // P in two bf16 terms (hi + lo) keeps ~16 mantissa bits.
        uint32_t h01, l01, h23, l23;
        rt::split_bf16x2(p0, p1, h01, l01);
        rt::split_bf16x2(p2, p3, h23, l23);
        const uint32_t bh0 = rt::movmatrix_trans(h01), bh1 = rt::movmatrix_trans(h23);
        const uint32_t bl0 = rt::movmatrix_trans(l01), bl1 = rt::movmatrix_trans(l23);

        // O^T += V^T P^T: 8 tiles of 16 dims; ldmatrix.trans of the V tile
        // gives the (dims x tokens) A fragments directly.
#pragma unroll
        for (int dd = 0; dd < 8; dd++) {
            const int c = ((dd & 3) << 1) + (mi & 1);
            const uint32_t addr =
                st + 4096u + (uint32_t)((dd >> 2) * 2048) + t_row + (uint32_t)((c ^ rr) << 4);
            uint32_t v[4];
            rt::ldsm_x4_trans(addr, v[0], v[1], v[2], v[3]);
            rt::mma_bf16_16816(o[dd], v, bh0, bh1);
            rt::mma_bf16_16816(o[dd], v, bl0, bl1);
        }
        __syncwarp();
            // Refill the stage: this item's next page, else the next item's.
            // After the first page the next item is set up - behind the
            // refill when this item still has pages to issue, so that its
            // loads wait with the ring full.
            const bool more = cur_iss < cur.n_mine;
            if (!have_nxt && !more)
                setup_next();
            if (more || nxt_iss < nxt.n_mine) {
                // The stage's shared memory was only read (ldmatrix, consumed
                // by the mma above) unless this was a tail page whose V rows
                // were zeroed: only generic writes need ordering before the
                // TMA write.
                if (valid < 16)
                    rt::fence_proxy_async_smem();
                if (more)
                    seq_issue(kv_map, a, cur, cur_iss++, issued++, stage0, bars, policy);
                else
                    seq_issue(kv_map, a, nxt, nxt_iss++, issued++, stage0, bars, policy);
            }
            if (!have_nxt)
                setup_next();
        }
        if (!have_nxt)
            setup_next();
        seq_finalize<G>(a, cur, o, m0, m1, l0, l1);
        id = id_n;
        cur = nxt;
        cur_iss = nxt_iss;
        // top the ring up with the new item's first pages (stages freed by
        // tail pages may hold generic writes)
        rt::fence_proxy_async_smem();
        for (; cur_iss < cur.n_mine && issued - used < (uint32_t)kStages; cur_iss++)
            seq_issue(kv_map, a, cur, cur_iss, issued++, stage0, bars, policy);
        __syncwarp();
    }
}

// One (group, row block, KV head, prefix chunk) item, processed by the whole
// CTA: the group's shared prefix pages stream once through the CTA's
// kWarps x kStages-stage ring (warp 0 loads the page ids, lane 0 issues the
// TMA copies), and each
// warp attends 16 query rows to every page - 16/G member sequences x G
// heads, so for G = 4 every row of the m16n8k16 tile is a real query (4
// sequences x 4 heads per warp, 16 sequences per CTA).  G = 8 needs two row
// blocks for 16 members; G = 1, 2 leave warps idle.  Each member's result is
// an unnormalised partial (o, max, sum) in slot `chunk` of its (b, h); the
// sequence kernel that runs next folds these into its own online softmax.
template <int G>
__device__ __forceinline__ bool process_group_item(const CUtensorMap &kv_map, const AttnArgs &a,
                                                   uint64_t gi, uint32_t n_live, uint32_t ring0,
                                                   uint64_t *gbars, uint32_t &gphases,
                                                   uint64_t policy, int32_t *s_pg,
                                                   uint32_t *s_cnt)
{
    constexpr int MPW = 16 / G;                        // member sequences per warp
    constexpr int RB = (16 * G + 16 * kWarps - 1) / (16 * kWarps);  // row blocks per group
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t Hkv = a.num_kv_heads, Hq = a.num_q_heads;
    const uint32_t g = (uint32_t)(gi % n_live);
    uint64_t rest = gi / n_live;
    const int rb = (int)(rest % RB);
    rest /= RB;
    const uint32_t h = (uint32_t)(rest % Hkv);
    const int chunk = (int)(rest / Hkv);
    const rt_attn_group_t &grp = a.groups[g];
    const uint32_t n_mem = min(grp.n_members, kMaxGroupMembers);
    const int P = (int)grp.shared_pages;
    const int cpg = (int)a.gchunk_pages;
    const int p0 = chunk * cpg;
    if (n_mem == 0 || P == 0 || p0 >= P)
        return true;
    const uint32_t src = grp.members[0];
    if (src >= a.num_seqs || (uint32_t)P > a.max_gchunks * (uint32_t)cpg ||
        (uint32_t)P > a.max_pages) {
        if (threadIdx.x == 0)
            flag_error(a.error, kErrGroup);
        return true;
    }
    const int np = min(P, p0 + cpg) - p0;

    // Every load of the prologue is one round trip behind the record: this
    // warp's query rows (from the record's member indices, clamped into
    // range and zeroed below if the member fails its checks), the members'
    // lengths and skips, and the chunk's page ids all go out together,
    // before the TMA issue (an asm statement the compiler does not move
    // loads across).
    // Rows of this warp: row r -> member (rb*kWarps + warp)*MPW + r/G, head r%G.
    const int wm0 = (rb * kWarps + warp) * MPW;
    const int rA = lane >> 2, rB = rA + 8, q4 = lane & 3;
    const int mA = wm0 + rA / G, mB = wm0 + rB / G;
    uint32_t bA = mA < (int)n_mem ? grp.members[mA] : a.num_seqs;
    uint32_t bB = mB < (int)n_mem ? grp.members[mB] : a.num_seqs;
    const bool inA = bA < a.num_seqs, inB = bB < a.num_seqs;
    if (!inA)
        bA = 0u;
    if (!inB)
        bB = 0u;
    const int LA = a.seq_lens[bA], LB = a.seq_lens[bB];
    const uint32_t kA = a.skip_pages[bA], kB = a.skip_pages[bB];
    uint32_t qf[8][4];
    {
        const uint32_t *qa = reinterpret_cast<const uint32_t *>(
            a.q + ((size_t)bA * Hq + (size_t)h * G + rA % G) * 128);
        const uint32_t *qb = reinterpret_cast<const uint32_t *>(
            a.q + ((size_t)bB * Hq + (size_t)h * G + rB % G) * 128);
#pragma unroll
        for (int j = 0; j < 8; j++) {
            qf[j][0] = qa[8 * j + q4];
            qf[j][1] = qb[8 * j + q4];
            qf[j][2] = qa[8 * j + 4 + q4];
            qf[j][3] = qb[8 * j + 4 + q4];
        }
    }

    // Page ids (warp 0): lane i holds pages i and 32 + i of this chunk.
    int pg_lo = 0, pg_hi = 0;
    if (warp == 0) {
        const int32_t *ptab = a.page_table + (size_t)src * a.max_pages + p0;
        if (lane < np)
            pg_lo = ptab[lane];
        if (lane + 32 < np)
            pg_hi = ptab[lane + 32];
        const bool bad = (lane < np && (pg_lo < 0 || (uint64_t)pg_lo >= a.arena_pages)) ||
                         (lane + 32 < np && (pg_hi < 0 || (uint64_t)pg_hi >= a.arena_pages));
        if (bad) {
            flag_error(a.error, kErrPage);
            if (pg_lo < 0 || (uint64_t)pg_lo >= a.arena_pages)
                pg_lo = 0;
            if (pg_hi < 0 || (uint64_t)pg_hi >= a.arena_pages)
                pg_hi = 0;
        }
    }
    // One page into its stage (a single thread).
    auto issue_page = [&](int i, int pg) {
        const int s = i % kGroupStages;
        const uint32_t bar = rt::smem_u32(&gbars[s]);
        const uint32_t dst = ring0 + (uint32_t)(s * kStageBytes);
        const int32_t row_k = (int32_t)(((int64_t)pg * Hkv + h) * 32);
        rt::mbar_arrive_expect_tx(bar, (uint32_t)kStageBytes);
        rt::tma_load_2d(dst, &kv_map, 0, row_k, bar, policy);
        rt::tma_load_2d(dst + 2048u, &kv_map, 64, row_k, bar, policy);
        rt::tma_load_2d(dst + 4096u, &kv_map, 0, row_k + 16, bar, policy);
        rt::tma_load_2d(dst + 6144u, &kv_map, 64, row_k + 16, bar, policy);
    };
    // When the chunk is longer than the ring, stages are refilled while the
    // item runs, by whichever warp finishes a stage last (below), so warp 0
    // puts the page ids in shared memory where every warp can read them.  No
    // barrier follows: a refill reads s_pg only after warp 0 has counted
    // itself done with that stage (its writes here come first in its program
    // order).
    const bool refill = np > kGroupStages;
    if (warp == 0 && refill) {
        s_pg[lane] = pg_lo;
        s_pg[lane + 32] = pg_hi;
    }
    // The ring's first pages, from warp 0.  (Spreading their issue over the
    // four warps started the pages sooner but lengthened the loop's pass by
    // 0.7%: the sequence kernel runs beside this one.)
    if (warp == 0) {
        for (int i = 0; i < np && i < kGroupStages; i++) {
            const int pg = __shfl_sync(0xffffffffu, i < 32 ? pg_lo : pg_hi, i & 31);
            if (lane == 0)
                issue_page(i, pg);
        }
    }

    // A member takes part when the group covers exactly its skipped pages.
    auto covers = [&](int L, uint32_t skip) -> bool {
        if (L < 0 || (uint32_t)L > a.max_seq_len || (uint32_t)L > a.max_pages * 16u)
            return false;
        return skip == (uint32_t)P && P <= ((L + 15) >> 4);
    };
    auto member_ok = [&](int m) -> bool {
        if (m >= (int)n_mem)
            return false;
        const uint32_t b = grp.members[m];
        return b < a.num_seqs && covers(a.seq_lens[b], a.skip_pages[b]);
    };
    const bool vA = inA && covers(LA, kA), vB = inB && covers(LB, kB);
    if (lane == 0 && chunk == 0 && h == 0)
        for (int m = wm0; m < wm0 + MPW && m < (int)n_mem; m++)
            if (!member_ok(m))
                flag_error(a.error, kErrGroup);
    const bool active = __any_sync(0xffffffffu, vA || vB);
#pragma unroll
    for (int j = 0; j < 8; j++) {
        if (!vA)
            qf[j][0] = qf[j][2] = 0u;
        if (!vB)
            qf[j][1] = qf[j][3] = 0u;
    }

    float o[16][4];
#pragma unroll
    for (int n = 0; n < 16; n++)
        o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.0f;
    float mA_run = -INFINITY, lA = 0.0f, mB_run = -INFINITY, lB = 0.0f;
    const int mi = lane >> 3, rr = lane & 7;
    const uint32_t k_row = (uint32_t)((((mi >> 1) << 3) + rr) * 128);
    const uint32_t v_row = (uint32_t)((((mi & 1) << 3) + rr) * 128);
    // The warps never wait for each other within the item: when the whole
    // chunk fits the ring every page is issued up front; otherwise each stage
    // is refilled by the last warp to finish reading it.
    for (int i = 0; i < np; i++) {
        const int s = i % kGroupStages;
        const bool ok = rt::mbar_wait_bounded(rt::smem_u32(&gbars[s]), (gphases >> s) & 1u,
                                              kWaitLimitNs);
        if (!__all_sync(0xffffffffu, ok)) {
            if (lane == 0)
                flag_error(a.error, kErrTimeout);
            // the caller stops the CTA; the copies issued so far are waited
            // for there (bounded), and warps still waiting on pages that will
            // not be refilled run into their own bounded waits
            return false;
        }
        gphases ^= 1u << s;
        if (active) {
            const uint32_t st = ring0 + (uint32_t)(s * kStageBytes);
            float sc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
            for (int j = 0; j < 8; j++) {
                const int c = ((j & 3) << 1) + (mi & 1);
                const uint32_t addr =
                    st + (uint32_t)((j >> 2) * 2048) + k_row + (uint32_t)((c ^ rr) << 4);
                uint32_t k0, k1, k2, k3;
                rt::ldsm_x4(addr, k0, k1, k2, k3);
                rt::mma_bf16_16816(sc[0], qf[j], k0, k1);
                rt::mma_bf16_16816(sc[1], qf[j], k2, k3);
            }
            // rows rA (c0, c1) and rB (c2, c3); every token of a shared page is valid
            const float a0 = sc[0][0] * a.scale_log2, a1 = sc[0][1] * a.scale_log2;
            const float a2 = sc[1][0] * a.scale_log2, a3 = sc[1][1] * a.scale_log2;
            const float b0 = sc[0][2] * a.scale_log2, b1 = sc[0][3] * a.scale_log2;
            const float b2 = sc[1][2] * a.scale_log2, b3 = sc[1][3] * a.scale_log2;
            float xa = fmaxf(fmaxf(a0, a1), fmaxf(a2, a3));
            float xb = fmaxf(fmaxf(b0, b1), fmaxf(b2, b3));
            xa = fmaxf(xa, __shfl_xor_sync(0xffffffffu, xa, 1));
            xa = fmaxf(xa, __shfl_xor_sync(0xffffffffu, xa, 2));
            xb = fmaxf(xb, __shfl_xor_sync(0xffffffffu, xb, 1));
            xb = fmaxf(xb, __shfl_xor_sync(0xffffffffu, xb, 2));
            const float nA = fmaxf(mA_run, xa), nB = fmaxf(mB_run, xb);
            const float cA = rt::fast_exp2(mA_run - nA), cB = rt::fast_exp2(mB_run - nB);
            const float pa0 = rt::fast_exp2(a0 - nA), pa1 = rt::fast_exp2(a1 - nA);
            const float pa2 = rt::fast_exp2(a2 - nA), pa3 = rt::fast_exp2(a3 - nA);
            const float pb0 = rt::fast_exp2(b0 - nB), pb1 = rt::fast_exp2(b1 - nB);
            const float pb2 = rt::fast_exp2(b2 - nB), pb3 = rt::fast_exp2(b3 - nB);
            lA = lA * cA + ((pa0 + pa1) + (pa2 + pa3));
            lB = lB * cB + ((pb0 + pb1) + (pb2 + pb3));
            mA_run = nA;
            mB_run = nB;
            // (skipped when no row of the warp found a new maximum: a factor
            // of exactly 1)
            if (!__all_sync(0xffffffffu, cA == 1.0f && cB == 1.0f)) {
#pragma unroll
                for (int n = 0; n < 16; n++) {
                    o[n][0] *= cA;
                    o[n][1] *= cA;
                    o[n][2] *= cB;
                    o[n][3] *= cB;
                }
            }
            uint32_t pf[4], pl[4];  // P = hi + lo in bf16 (as in the sequence items)
            rt::split_bf16x2(pa0, pa1, pf[0], pl[0]);
            rt::split_bf16x2(pb0, pb1, pf[1], pl[1]);
            rt::split_bf16x2(pa2, pa3, pf[2], pl[2]);
            rt::split_bf16x2(pb2, pb3, pf[3], pl[3]);
#pragma unroll
            for (int dd = 0; dd < 8; dd++) {
                const int c = ((dd & 3) << 1) + (mi >> 1);
                const uint32_t addr =
                    st + 4096u + (uint32_t)((dd >> 2) * 2048) + v_row + (uint32_t)((c ^ rr) << 4);
                uint32_t v0, v1, v2, v3;
                rt::ldsm_x4_trans(addr, v0, v1, v2, v3);
                rt::mma_bf16_16816(o[2 * dd], pf, v0, v1);
                rt::mma_bf16_16816(o[2 * dd + 1], pf, v2, v3);
                rt::mma_bf16_16816(o[2 * dd], pl, v0, v1);
                rt::mma_bf16_16816(o[2 * dd + 1], pl, v2, v3);
            }
        }
        if (refill) {
            // The warp is done with stage s (shared-memory reads only, so the
            // TMA rewrite needs no proxy fence); the fourth warp to say so
            // resets the count and refills the stage with page i + stages.
            __syncwarp();
            if (lane == 0) {
                __threadfence_block();
                if (atomicAdd(&s_cnt[s], 1u) == (uint32_t)kWarps - 1u) {
                    __threadfence_block();  // every warp's count, warp 0's s_pg, then the read
                    s_cnt[s] = 0u;
                    if (i + kGroupStages < np)
                        issue_page(i + kGroupStages, s_pg[i + kGroupStages]);
                }
            }
        }
    }
    if (!active)
        return true;
    lA += __shfl_xor_sync(0xffffffffu, lA, 1);
    lA += __shfl_xor_sync(0xffffffffu, lA, 2);
    lB += __shfl_xor_sync(0xffffffffu, lB, 1);
    lB += __shfl_xor_sync(0xffffffffu, lB, 2);

    // Partials of both rows of this lane; the kernel boundary publishes them.
    if (vA) {
        const size_t pi = (((size_t)bA * Hkv + h) * a.slots + chunk) * G + rA % G;
        float *dst = a.part_o + pi * 128 + 2 * q4;
#pragma unroll
        for (int n = 0; n < 16; n++)
            *reinterpret_cast<float2 *>(dst + n * 8) = make_float2(o[n][0], o[n][1]);
        if (q4 == 0)
            *reinterpret_cast<float2 *>(a.part_ml + pi * 2) = make_float2(mA_run, lA);
    }
    if (vB) {
        const size_t pi = (((size_t)bB * Hkv + h) * a.slots + chunk) * G + rB % G;
        float *dst = a.part_o + pi * 128 + 2 * q4;
#pragma unroll
        for (int n = 0; n < 16; n++)
            *reinterpret_cast<float2 *>(dst + n * 8) = make_float2(o[n][2], o[n][3]);
        if (q4 == 0)
            *reinterpret_cast<float2 *>(a.part_ml + pi * 2) = make_float2(mB_run, lB);
    }
    return true;
}

// Shared-prefix kernel of the grouped entry point: persistent CTAs take
// (group, row block, head, chunk) items from a dispenser; the last CTA out
// resets it for the next launch.
template <int G>
__global__ void __launch_bounds__(kWarps * 32, kGroupCtasPerSm)
paged_gqa_group_kernel(const __grid_constant__ CUtensorMap kv_map, const AttnArgs a)
{
    extern __shared__ uint8_t smem_raw[];
    __shared__ __align__(8) uint64_t gbars[kGroupStages];
    __shared__ unsigned long long s_gitem;
    __shared__ int32_t s_pg[kMaxChunkPages];        // page ids of the current item
    __shared__ uint32_t s_cnt[kGroupStages];        // warps done with each stage
    const uint32_t raw_u32 = rt::smem_u32(smem_raw);
    const uint32_t base_u32 = (raw_u32 + 1023u) & ~1023u;  // 128-byte swizzle: 1 KiB aligned
    if (threadIdx.x == 0) {
        rt::prefetch_tensormap(&kv_map);
        for (int s = 0; s < kGroupStages; s++) {
            rt::mbar_init(rt::smem_u32(&gbars[s]), 1u);
            s_cnt[s] = 0u;
        }
        rt::mbar_fence_init();
    }
    __syncthreads();
    // Launched as a programmatic dependent of the kernel that wrote the
    // queries and tables: wait for it before reading anything.
    rt::grid_dep_wait();
    // The sequence kernel may start on SMs this grid leaves free; it waits
    // for this grid's completion before it reads the partials.
    rt::grid_dep_launch();
    // Shared prefix pages are read again by the next pass's group items: keep
    // them in L2 ahead of the sequences' private pages (config 5 +0.7%).
    const uint64_t policy = a.evict_first ? rt::l2_policy_evict_first() : rt::l2_policy_evict_last();
    constexpr int RB = (16 * G + 16 * kWarps - 1) / (16 * kWarps);
    const uint32_t n_live = min(*a.n_groups, a.max_groups);
    const uint64_t n_gi = (uint64_t)n_live * RB * a.num_kv_heads * a.max_gchunks;
    uint32_t gphases = 0;
    // The first item is the CTA's own index (no dispenser round trip before
    // its first page); further items come from the dispenser, counted from
    // gridDim.x.
    bool first = true;
    while (n_gi) {
        uint64_t gi = blockIdx.x;
        if (!first) {
            if (threadIdx.x == 0)
                s_gitem = gridDim.x + atomicAdd(a.group_next, 1ull);
            __syncthreads();
            gi = s_gitem;
            __syncthreads();
        }
        first = false;
        if (gi >= n_gi)
            break;
        // A false return means a wait expired (flagged): stop taking items,
        // after giving the copies still in flight a bounded chance to land.
        const bool ok = process_group_item<G>(kv_map, a, gi, n_live, base_u32, gbars, gphases, policy,
                                              s_pg, s_cnt);
        if (!__syncthreads_and(ok)) {
            if (threadIdx.x == 0)
                for (int st = 0; st < kGroupStages; st++)
                    (void)rt::mbar_wait_bounded(rt::smem_u32(&gbars[st]), (gphases >> st) & 1u,
                                                kWaitLimitNs / 64);
            break;
        }
    }
    if (threadIdx.x == 0) {
        __threadfence();
        if (atomicAdd(a.group_done, 1u) == gridDim.x - 1u) {
            *a.group_next = 0ull;
            *a.group_done = 0u;
            __threadfence();
        }
    }
}

// Persistent warps take items in increasing order from a global dispenser
// (one atomic per item, fetched one item ahead), so a warp whose item is
// empty moves on at once, long and short items balance dynamically, and the
// items of a GRPO group's sequences run side by side.  The last warp to
// leave resets the dispenser for the next launch.
template <int G>
__global__ void __launch_bounds__(kWarps * 32, kCtasPerSm)
paged_gqa_decode_kernel(const __grid_constant__ CUtensorMap kv_map, const AttnArgs a)
{
    extern __shared__ uint8_t smem_raw[];
    __shared__ __align__(8) uint64_t bars[kWarps][kStages];

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // 1 KiB-aligned stage ring of this warp (128-byte swizzle repeats every 1 KiB).
    const uint32_t raw_u32 = rt::smem_u32(smem_raw);
    const uint32_t base_u32 = (raw_u32 + 1023u) & ~1023u;
    uint8_t *base_ptr = smem_raw + (base_u32 - raw_u32);
    const uint32_t stage0 = base_u32 + (uint32_t)(warp * kStages * kStageBytes);

    if (threadIdx.x == 0 && blockIdx.x == 0)
        *a.n_counters = a.num_seqs * a.num_kv_heads;
    if (lane == 0) {
        rt::prefetch_tensormap(&kv_map);
        for (int s = 0; s < kStages; s++)
            rt::mbar_init(rt::smem_u32(&bars[warp][s]), 1u);
        rt::mbar_fence_init();
        rt::fence_proxy_async_smem();
    }
    __syncwarp();
    // The next kernel of the stream (launched as a programmatic dependent)
    // may be scheduled once every CTA of this grid has started.
    rt::grid_dep_launch();
    const uint64_t policy = a.evict_first ? rt::l2_policy_evict_first() : rt::l2_policy_evict_normal();
    // this warp's query-row buffer, after the CTA's stage rings
    uint32_t *qs = reinterpret_cast<uint32_t *>(base_ptr + kWarps * kStages * kStageBytes) +
                   warp * G * kQRowWords;
    __shared__ uint32_t s_pre[kPlanSeqs];
    const SeqPlan pl = seq_plan(a, s_pre);
    run_seq_items<G>(kv_map, a, pl, stage0, base_ptr, base_u32, bars[warp], policy, qs);
    if (lane == 0) {
        __threadfence();
        const unsigned int total = gridDim.x * kWarps;
        if (atomicAdd(a.work_done, 1u) == total - 1u) {
            *a.work_next = 0ull;
            *a.work_done = 0u;
            __threadfence();
        }
    }
}

// ------------------------------------------------------------------ host
struct Plan {
    uint32_t group, chunk_pages, max_chunks;
    uint32_t gchunk_pages, max_gchunks, slots;  // group phase (0 when ungrouped)
    size_t off_counters, off_ml, off_o, total;
};

#ifndef RT_ATTN_GROUP_CHUNK_PAGES
#define RT_ATTN_GROUP_CHUNK_PAGES 16
#endif
constexpr uint32_t kDefaultGroupChunkPages = RT_ATTN_GROUP_CHUNK_PAGES;

// Workspace header: error word at 0, per-warp item dispenser at 8/16, group
// item dispenser at 24/32, number of arrival counters of the last call at 40
// (written by the sequence kernel); arrival counters from 256.
int make_plan(const rt_attn_params_t *p, Plan *pl, const rt_attn_group_params_t *gp = nullptr)
{
    if (!p) {
        rt::set_error("attention: null params");
        return RT_EINVAL;
    }
    if (p->head_dim != 128u) {
        rt::set_error("attention: head_dim must be 128 (got %u)", p->head_dim);
        return RT_EINVAL;
    }
    if (p->num_kv_heads == 0 || p->num_q_heads % p->num_kv_heads) {
        rt::set_error("attention: num_q_heads %u not a multiple of num_kv_heads %u",
                      p->num_q_heads, p->num_kv_heads);
        return RT_EINVAL;
    }
    const uint32_t g = p->num_q_heads / p->num_kv_heads;
    if (g != 1 && g != 2 && g != 4 && g != 8) {
        rt::set_error("attention: group size %u unsupported (1, 2, 4 or 8)", g);
        return RT_EINVAL;
    }
    if (p->num_seqs == 0 || p->num_kv_heads > 65535u) {
        rt::set_error("attention: num_seqs %u / num_kv_heads %u out of range", p->num_seqs,
                      p->num_kv_heads);
        return RT_EINVAL;
    }
    if (p->max_pages_per_seq == 0 || p->max_seq_len > p->max_pages_per_seq * 16u) {
        rt::set_error("attention: max_seq_len %u exceeds page capacity %u x 16", p->max_seq_len,
                      p->max_pages_per_seq);
        return RT_EINVAL;
    }
    const uint32_t pages_max = (p->max_seq_len + 15u) / 16u;
    uint32_t cp = p->chunk_pages;
    if (cp == 0) {
        // Up to 48 pages (768 tokens) per warp item, halved while there are
        // fewer than two items per warp slot of the GPU: the ragged config-2
        // batch and the rollout loop both land on 24 (config 2: 5,418 GB/s
        // against 4,695 with 48-page items, 3 CTAs x 4 warps per SM).
        cp = 48;
        const uint64_t warp_slots = (uint64_t)rt::num_sms() * kCtasPerSm * kWarps;
        while (cp > 4 && (uint64_t)p->num_seqs * p->num_kv_heads * ((pages_max + cp - 1) / cp) <
                             2u * warp_slots)
            cp /= 2;
    }
    if (cp < 1 || cp > (uint32_t)kMaxChunkPages) {
        rt::set_error("attention: chunk_pages %u outside 1..%d", cp, kMaxChunkPages);
        return RT_EINVAL;
    }
    pl->group = g;
    pl->chunk_pages = cp;
    pl->max_chunks = pages_max ? (pages_max + cp - 1) / cp : 1u;
    pl->gchunk_pages = 0;
    pl->max_gchunks = 0;
    if (gp) {
        // Auto: 16-page items; 32 when prefixes can be long (max_shared_pages
        // > 64), where 16-page items multiply the per-item prologue (config
        // 4's 1,024-token base + prompt: 119 against 109 us of attention per
        // pass), while short prefixes need the smaller items to fill the GPU.
        uint32_t cpg = gp->chunk_pages ? gp->chunk_pages
                                       : (gp->max_shared_pages > 64u ? 2u * kDefaultGroupChunkPages
                                                                      : kDefaultGroupChunkPages);
        if (gp->max_groups == 0 || gp->max_groups > (1u << 24) || cpg > (uint32_t)kMaxChunkPages ||
            gp->max_shared_pages > pages_max) {
            rt::set_error("attention: group params out of range (max_groups %u, "
                          "max_shared_pages %u of %u pages, chunk_pages %u)",
                          gp->max_groups, gp->max_shared_pages, pages_max, cpg);
            return RT_EINVAL;
        }
        pl->gchunk_pages = cpg;
        pl->max_gchunks = (gp->max_shared_pages + cpg - 1) / cpg;
    }
    pl->slots = pl->max_gchunks + pl->max_chunks;
    const size_t bh = (size_t)p->num_seqs * p->num_kv_heads;
    auto up = [](size_t x) { return (x + 255u) & ~(size_t)255u; };
    pl->off_counters = 256;
    pl->off_ml = pl->off_counters + up(bh * 4u);
    pl->off_o = pl->off_ml + up(bh * pl->slots * g * 2u * 4u);
    pl->total = pl->off_o + up(bh * pl->slots * g * 128u * 4u);
    return RT_OK;
}

struct MapCacheEntry {
    const void *base;
    uint64_t rows;
    CUtensorMap map;
};

int get_kv_map(const void *base, uint64_t rows, CUtensorMap *out)
{
    static std::mutex mu;
    static MapCacheEntry cache[8];
    static int next = 0;
    std::lock_guard<std::mutex> lk(mu);
    for (auto &e : cache)
        if (e.base == base && e.rows == rows) {
            *out = e.map;
            return RT_OK;
        }
    MapCacheEntry &e = cache[next];
    int rc = rt::encode_kv_rows_map(&e.map, base, rows);
    if (rc != RT_OK) {
        e.base = nullptr;
        return rc;
    }
    e.base = base;
    e.rows = rows;
    next = (next + 1) % 8;
    *out = e.map;
    return RT_OK;
}

// Opt-in to > 48 KiB dynamic shared memory, once per device and group size.
template <int G>
int prepare_g()
{
    static std::mutex mu;
    static bool done[64] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess)
        return rt::cuda_fail(e, "attention: cudaGetDevice");
    std::lock_guard<std::mutex> lk(mu);
    if (dev < 64 && done[dev])
        return RT_OK;
    e = cudaFuncSetAttribute(paged_gqa_decode_kernel<G>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             seq_smem_bytes<G>());
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(paged_gqa_group_kernel<G>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, kGroupSmemBytes);
    if (e != cudaSuccess)
        return rt::cuda_fail(e, "attention: cudaFuncSetAttribute");
    if (dev < 64)
        done[dev] = true;
    return RT_OK;
}

int prepare_group(uint32_t g)
{
    switch (g) {
    case 1: return prepare_g<1>();
    case 2: return prepare_g<2>();
    case 4: return prepare_g<4>();
    default: return prepare_g<8>();
    }
}

template <int G>
int launch_g(const CUtensorMap &map, const AttnArgs &args, dim3 grid, cudaStream_t s)
{
    int rc = prepare_g<G>();
    if (rc != RT_OK)
        return rc;
    if (!args.groups) {
        paged_gqa_decode_kernel<G><<<grid, kWarps * 32, seq_smem_bytes<G>(), s>>>(map, args);
        cudaError_t e = cudaGetLastError();
        return e == cudaSuccess ? RT_OK : rt::cuda_fail(e, "attention: launch");
    }
    // Group prefixes first.  The sequence kernel is a programmatic dependent
    // launch: its CTAs start on SMs the group grid frees and run their own
    // prologue and suffix pages; each waits for the group grid (griddepcontrol)
    // only before folding in the prefix partials.
    // The group kernel itself is a programmatic dependent of whatever ran
    // before it (it waits for that kernel before reading its inputs).
    cudaLaunchAttribute pdl[1];
    pdl[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    pdl[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t gcfg = {};
    gcfg.gridDim = dim3((unsigned)rt::num_sms() * kGroupCtasPerSm);
    gcfg.blockDim = dim3(kWarps * 32);
    gcfg.dynamicSmemBytes = kGroupSmemBytes;
    gcfg.stream = s;
    gcfg.attrs = pdl;
    gcfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&gcfg, paged_gqa_group_kernel<G>, map, args);
    if (e != cudaSuccess)
        return rt::cuda_fail(e, "attention: group launch");
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(kWarps * 32);
    cfg.dynamicSmemBytes = seq_smem_bytes<G>();
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, paged_gqa_decode_kernel<G>, map, args);
    return e == cudaSuccess ? RT_OK : rt::cuda_fail(e, "attention: launch");
}

}  // namespace

int rt::attn_prepare(const rt_attn_params_t *p)
{
    Plan pl;
    int rc = make_plan(p, &pl);
    return rc == RT_OK ? prepare_group(pl.group) : rc;
}

extern "C" size_t rt_attn_workspace_bytes(const rt_attn_params_t *p)
{
    Plan pl;
    return make_plan(p, &pl) == RT_OK ? pl.total : 0;
}

extern "C" int rt_attn_workspace_init(void *ws, size_t bytes, void *stream)
{
    if (!ws) {
        rt::set_error("attention: null workspace");
        return RT_EINVAL;
    }
    cudaError_t e = cudaMemsetAsync(ws, 0, bytes, (cudaStream_t)stream);
    return e == cudaSuccess ? RT_OK : rt::cuda_fail(e, "attention: workspace memset");
}

extern "C" int rt_attn_plan(const rt_attn_params_t *p, uint32_t *chunk_pages, uint32_t *max_chunks,
                            uint64_t *ctas)
{
    Plan pl;
    int rc = make_plan(p, &pl);
    if (rc != RT_OK)
        return rc;
    if (chunk_pages) *chunk_pages = pl.chunk_pages;
    if (max_chunks) *max_chunks = pl.max_chunks;
    if (ctas) {
        const uint64_t need = ((uint64_t)pl.max_chunks * p->num_kv_heads * p->num_seqs + kWarps - 1) / kWarps;
        const uint64_t resident = (uint64_t)rt::num_sms() * kCtasPerSm;
        *ctas = need < resident ? need : resident;
    }
    return RT_OK;
}

namespace {

int launch_attention(const rt_attn_params_t *p, const rt_attn_group_params_t *gp, const void *q,
                     const void *kv_arena, const int32_t *page_table, const int32_t *seq_lens,
                     const rt_attn_group_t *groups, const uint32_t *n_groups,
                     const uint32_t *skip_pages, float *out, void *workspace,
                     size_t workspace_bytes, void *stream, const uint32_t *dyn_chunks = nullptr)
{
    Plan pl;
    int rc = make_plan(p, &pl, gp);
    if (rc != RT_OK)
        return rc;
    if (!q || !kv_arena || !page_table || !seq_lens || !out || !workspace) {
        rt::set_error("attention: null pointer argument");
        return RT_EINVAL;
    }
    if (gp && (!groups || !n_groups || !skip_pages)) {
        rt::set_error("attention: grouped call needs groups, n_groups and skip_pages");
        return RT_EINVAL;
    }
    if (((uintptr_t)q & 3u) || ((uintptr_t)out & 3u) || ((uintptr_t)workspace & 255u) ||
        ((uintptr_t)kv_arena & 15u) || ((uintptr_t)page_table & 3u) ||
        ((uintptr_t)seq_lens & 3u) || ((uintptr_t)groups & 3u) || ((uintptr_t)n_groups & 3u) ||
        ((uintptr_t)skip_pages & 3u)) {
        rt::set_error("attention: misaligned pointer (q/out/tables 4 B, arena 16 B, workspace 256 B)");
        return RT_EINVAL;
    }
    if (workspace_bytes < pl.total) {
        rt::set_error("attention: workspace %zu B < required %zu B", workspace_bytes, pl.total);
        return RT_ENOMEM;
    }
    if (p->arena_pages == 0 || p->arena_pages > (1ull << 31) / (32ull * p->num_kv_heads)) {
        rt::set_error("attention: arena_pages %llu out of range",
                      (unsigned long long)p->arena_pages);
        return RT_EINVAL;
    }
    CUtensorMap map;
    rc = get_kv_map(kv_arena, p->arena_pages * p->num_kv_heads * 32u, &map);
    if (rc != RT_OK)
        return rc;

    uint8_t *ws = static_cast<uint8_t *>(workspace);
    AttnArgs args;
    args.q = static_cast<const __nv_bfloat16 *>(q);
    args.page_table = page_table;
    args.seq_lens = seq_lens;
    args.out = out;
    args.part_o = reinterpret_cast<float *>(ws + pl.off_o);
    args.part_ml = reinterpret_cast<float *>(ws + pl.off_ml);
    args.counters = reinterpret_cast<int32_t *>(ws + pl.off_counters);
    args.error = reinterpret_cast<int32_t *>(ws);
    args.n_counters = reinterpret_cast<uint32_t *>(ws + 40);
    args.work_next = reinterpret_cast<unsigned long long *>(ws + 8);
    args.work_done = reinterpret_cast<unsigned int *>(ws + 16);
    args.num_q_heads = p->num_q_heads;
    args.num_kv_heads = p->num_kv_heads;
    args.max_pages = p->max_pages_per_seq;
    args.max_chunks = pl.max_chunks;
    args.chunk_pages = pl.chunk_pages;
    args.max_seq_len = p->max_seq_len;
    args.arena_pages = p->arena_pages;
    args.scale_log2 = p->scale * 1.4426950408889634f;
    args.evict_first = p->kv_evict_first ? 1u : 0u;
    args.num_seqs = p->num_seqs;
    args.n_items = (uint64_t)p->num_seqs * p->num_kv_heads * pl.max_chunks;
    args.groups = gp ? groups : nullptr;
    args.n_groups = gp ? n_groups : nullptr;
    args.skip_pages = gp ? skip_pages : nullptr;
    args.group_next = reinterpret_cast<unsigned long long *>(ws + 24);
    args.group_done = reinterpret_cast<unsigned int *>(ws + 32);
    args.max_groups = gp ? gp->max_groups : 0u;
    args.gchunk_pages = gp ? pl.gchunk_pages : 1u;
    args.max_gchunks = pl.max_gchunks;
    args.slots = pl.slots;
    args.dyn_chunks = dyn_chunks;
    // Persistent grid: kCtasPerSm CTAs per SM (the shared-memory limit), never
    // more CTAs than there are items to hand out.
    uint64_t ctas = (args.n_items + kWarps - 1) / kWarps;
    const uint64_t resident = (uint64_t)rt::num_sms() * kCtasPerSm;
    if (ctas > resident)
        ctas = resident;
    const dim3 grid((unsigned)ctas);
    cudaStream_t s = (cudaStream_t)stream;
    switch (pl.group) {
    case 1: return launch_g<1>(map, args, grid, s);
    case 2: return launch_g<2>(map, args, grid, s);
    case 4: return launch_g<4>(map, args, grid, s);
    default: return launch_g<8>(map, args, grid, s);
    }
}

}  // namespace

extern "C" int rt_paged_decode_attention(const rt_attn_params_t *p, const void *q,
                                         const void *kv_arena, const int32_t *page_table,
                                         const int32_t *seq_lens, float *out, void *workspace,
                                         size_t workspace_bytes, void *stream)
{
    return launch_attention(p, nullptr, q, kv_arena, page_table, seq_lens, nullptr, nullptr,
                            nullptr, out, workspace, workspace_bytes, stream);
}

extern "C" size_t rt_attn_grouped_workspace_bytes(const rt_attn_params_t *p,
                                                  const rt_attn_group_params_t *gp)
{
    Plan pl;
    if (!gp)
        return rt_attn_workspace_bytes(p);
    return make_plan(p, &pl, gp) == RT_OK ? pl.total : 0;
}

extern "C" int rt_paged_decode_attention_grouped(
    const rt_attn_params_t *p, const rt_attn_group_params_t *gp, const void *q,
    const void *kv_arena, const int32_t *page_table, const int32_t *seq_lens,
    const rt_attn_group_t *groups, const uint32_t *n_groups, const uint32_t *skip_pages,
    float *out, void *workspace, size_t workspace_bytes, void *stream)
{
    if (!gp) {
        rt::set_error("attention: null group params");
        return RT_EINVAL;
    }
    return launch_attention(p, gp, q, kv_arena, page_table, seq_lens, groups, n_groups,
                            skip_pages, out, workspace, workspace_bytes, stream);
}

int rt::attn_launch(const rt_attn_params_t *p, const rt_attn_group_params_t *gp, const void *q,
                    const void *kv_arena, const int32_t *page_table, const int32_t *seq_lens,
                    const rt_attn_group_t *groups, const uint32_t *n_groups,
                    const uint32_t *skip_pages, float *out, void *workspace,
                    size_t workspace_bytes, const uint32_t *dyn_chunks, cudaStream_t stream)
{
    return launch_attention(p, gp, q, kv_arena, page_table, seq_lens, groups, n_groups,
                            skip_pages, out, workspace, workspace_bytes, stream, dyn_chunks);
}

int rt::attn_item_shape(const rt_attn_params_t *p, const rt_attn_group_params_t *gp,
                        uint32_t *chunk_pages, uint32_t *gchunk_pages, uint32_t *max_gchunks)
{
    Plan pl;
    const int rc = make_plan(p, &pl, gp);
    if (rc != RT_OK)
        return rc;
    *chunk_pages = pl.chunk_pages;
    *gchunk_pages = gp ? pl.gchunk_pages : 1u;
    *max_gchunks = pl.max_gchunks;
    return RT_OK;
}

extern "C" int rt_attn_workspace_error(void *workspace, void *stream, int32_t *code)
{
    if (!workspace || !code) {
        rt::set_error("attention: null argument");
        return RT_EINVAL;
    }
    uint32_t hdr[12] = {};
    cudaStream_t s = (cudaStream_t)stream;
    cudaError_t e = cudaMemcpyAsync(hdr, workspace, sizeof(hdr), cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess)
        e = cudaStreamSynchronize(s);
    if (e == cudaSuccess)
        e = cudaMemsetAsync(workspace, 0, 4, s);
    // A failed call may have left arrival counters part-counted.
    if (e == cudaSuccess && hdr[0] != 0u && hdr[10] != 0u)
        e = cudaMemsetAsync(static_cast<uint8_t *>(workspace) + 256, 0, (size_t)hdr[10] * 4u, s);
    if (e != cudaSuccess)
        return rt::cuda_fail(e, "attention: read error word");
    *code = (int32_t)hdr[0];
    return RT_OK;
}

// ---------------------------------------------------------------------------
// Allocation-free variant.  Some callers cannot create device memory at the
// point where they run decode attention: code that follows a no-allocation
// hot-path rule (the reference's own HotpathGuard counts every allocation
// made after activation as a violation), hosts whose device memory is owned
// by another allocator that must not be bypassed, and loops where a
// cudaMalloc/cudaFree would synchronise the device.  For them the split-K
// scratch is a fixed array in the library's own device memory instead of a
// caller-provided workspace.
namespace {

constexpr size_t kStaticScratchBytes = (size_t)32 << 20;  // 32 MiB per device
__device__ __align__(256) uint8_t g_attn_static_scratch[kStaticScratchBytes];

// Device address of g_attn_static_scratch, resolved once per device and
// context.  In host code the symbol names a host-side stand-in, not device
// memory, so the kernels must be given this address.  The cache is keyed by
// the driver's context id as well as the device, so a context created after
// cudaDeviceReset (where the library's module, and the array, are loaded
// afresh) gets its own lookup instead of a stale address.
typedef int (*ctx_get_current_fn)(void **ctx);
typedef int (*ctx_get_id_fn)(void *ctx, unsigned long long *id);

// Id of the calling thread's current context; false when none is current
// yet (before the first runtime call on the device) or the driver entry
// points are unavailable.
bool current_context_id(unsigned long long *id)
{
    static ctx_get_current_fn get_current = nullptr;
    static ctx_get_id_fn get_id = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_current = reinterpret_cast<ctx_get_current_fn>(f);
        f = nullptr;
        if (cudaGetDriverEntryPoint("cuCtxGetId", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_id = reinterpret_cast<ctx_get_id_fn>(f);
    });
    void *ctx = nullptr;
    return get_current && get_id && get_current(&ctx) == 0 && ctx && get_id(ctx, id) == 0;
}

int static_scratch_ptr(void **out)
{
    static std::mutex mu;
    static void *ptrs[64] = {};
    static unsigned long long ctx_ids[64] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess)
        return rt::cuda_fail(e, "attention_noalloc: cudaGetDevice");
    if (dev < 0 || dev >= 64) {
        rt::set_error("attention_noalloc: device index %d out of range", dev);
        return RT_EINVAL;
    }
    unsigned long long ctx = 0;
    const bool have_ctx = current_context_id(&ctx);
    std::lock_guard<std::mutex> lk(mu);
    if (!have_ctx || !ptrs[dev] || ctx_ids[dev] != ctx) {
        // The lookup also initialises the device's context when none is
        // current yet; the id is read after it in that case.
        void *p = nullptr;
        e = cudaGetSymbolAddress(&p, g_attn_static_scratch);
        if (e != cudaSuccess)
            return rt::cuda_fail(e, "attention_noalloc: cudaGetSymbolAddress");
        if (!have_ctx && !current_context_id(&ctx)) {
            rt::set_error("attention_noalloc: cannot identify the current CUDA context");
            return RT_ECUDA;
        }
        ptrs[dev] = p;
        ctx_ids[dev] = ctx;
    }
    *out = ptrs[dev];
    return RT_OK;
}

}  // namespace

extern "C" int rt_paged_decode_attention_noalloc(const rt_attn_params_t *p, const void *q,
                                                 const void *kv_arena, const int32_t *page_table,
                                                 const int32_t *seq_lens, float *out,
                                                 void *stream)
{
    Plan pl;
    int rc = make_plan(p, &pl);
    if (rc != RT_OK)
        return rc;
    if (pl.total > kStaticScratchBytes) {
        rt::set_error("attention_noalloc: these shapes need %zu B of scratch, the built-in "
                      "array holds %zu B; use rt_paged_decode_attention with a workspace",
                      pl.total, kStaticScratchBytes);
        return RT_ENOMEM;
    }
    void *scratch = nullptr;
    rc = static_scratch_ptr(&scratch);
    if (rc != RT_OK)
        return rc;
    // The error word and the split-K arrival counters must start at zero;
    // the array keeps whatever the previous call left in it.
    cudaError_t e = cudaMemsetAsync(scratch, 0, pl.off_ml, (cudaStream_t)stream);
    if (e != cudaSuccess)
        return rt::cuda_fail(e, "attention_noalloc: clear counters");
    return rt_paged_decode_attention(p, q, kv_arena, page_table, seq_lens, out, scratch,
                                     kStaticScratchBytes, stream);
}

extern "C" int rt_paged_decode_attention_noalloc_error(int32_t *code, void *stream)
{
    if (!code) {
        rt::set_error("attention_noalloc_error: null code");
        return RT_EINVAL;
    }
    void *scratch = nullptr;
    const int rc = static_scratch_ptr(&scratch);
    if (rc != RT_OK)
        return rc;
    return rt_attn_workspace_error(scratch, stream, code);
}
