// decode_worker.cu - the per-step CommandRing decode path on sm_100a.
//
// Reference: cu/worker.cu:25-131 (decode_worker, process_descriptor) and
// cu/attention_decode.cu:16-204 (decode_synth_query_component,
// decode_load_query, attention_decode_step_fixed128).
//
// Reference shape: one persistent warp per SM, each lane 0 polling the
// single-consumer CommandRing and pushing to the single-producer
// CompletionRing, so 148 warps race on both rings.  Here the rings keep
// their one-consumer / one-producer contracts:
//
//   pump warp (CTA 0, warp 0)
//     takes up to 256 ring records per pass with all reads in flight at
//     once (whole 512-byte spans per warp instruction: one host-link round
//     trip per batch, not one per record), reads prod.tail only when the
//     last value seen cannot fill a batch, copies the work into a device
//     queue, releases cons.head once per batch, and stops at the
//     stop_sentinels-th UINT64_MAX sentinel.  While a batch's reads are in
//     flight it delivers finished completions to the CompletionRing in
//     ring order, up to a batch per tail release.
//   worker warps (every other warp of the grid)
//     claim queue tickets with an atomic, stage the descriptor's KV rows
//     into their own shared-memory stage with a bulk async copy (mbarrier
//     completion), run the fixed128 step and publish the completion.
//
// The step reproduces the reference kernel's fp32 evaluation order, so
// outputs and token ids are identical to it: a token's score is eight
// ascending-d fma chains (d = i mod 8) combined as
// ((p0+p4)+(p2+p6))+((p1+p5)+(p3+p7)) and scaled by rsqrtf(128); online
// softmax over 16-token tiles with the tile norm summed in token order and
// norm' = fma(norm, rescale, tile_norm); out[d] = fma chains over the
// tile's tokens starting from out[d] * rescale; a final division by the
// norm.  Ties of the argmax go to the lowest d mod 32, then the lowest
// d / 32 (the reference's lane-then-stride scan).
//
// Every wait is bounded: the pump gives up after idle_timeout_ms without
// progress, workers after that plus a margin, the KV copy after 1 s; each
// sets an error word instead of hanging.
#include <cuda_fp16.h>
#include <math.h>
#include <mutex>
#include <stdint.h>
#include <string.h>

#include "attention_decode.h"
#include "rlrt.h"
#include "rt_common.cuh"

namespace {

constexpr uint32_t kQueue = 4096;        // device work-queue entries (power of two)
constexpr uint32_t kPumpBatch = 256;     // ring records taken per pump pass
constexpr uint32_t kWarpsPerCta = 4;
constexpr uint32_t kKvBytes = KV_LAYOUT_BLOCK_BYTES;          // 16 KiB: K plane, V plane
constexpr uint32_t kVPlane = KV_LAYOUT_K_BYTES;               // 8 KiB
constexpr uint32_t kRowBytes = KV_LAYOUT_HEAD_DIM * 2u;       // 256 B per token row
constexpr uint32_t kStageBytes = kKvBytes + 512u + 128u;      // KV + q fp32[128] + mbarrier
constexpr uint64_t kCopyLimitNs = 1000000000ull;              // 1 s for one 16 KiB copy
constexpr uint64_t kWorkerMarginNs = 5000000000ull;

static_assert(kStageBytes % 128u == 0u, "stages stay 128-byte aligned");
static_assert(sizeof(Descriptor) == 32 && sizeof(Completion) == 32, "32-byte ring records");

struct alignas(128) Line {
    uint32_t v;
    uint32_t pad[31];
};

// Device control block of one decode-worker launch.
struct DwCtl {
    Line published;  // work descriptors in the queue (monotonic, modulo 2^32)
    Line stop;       // 1: `published` is final
    Line claimed;    // queue tickets handed to worker warps
    Line drained;    // completions delivered to the CompletionRing
    unsigned long long consumed;  // ring records taken, sentinels included
    unsigned long long completed;
    uint32_t sentinels;
    uint32_t comp_full;
    int32_t error;
    uint32_t bad_block;
    uint32_t workers;
    uint32_t finished;
};

struct DwQueue {
    uint4 desc[kQueue * 2];
    uint4 comp[kQueue * 2];
    uint32_t ready[kQueue];  // ticket + 1 once comp[ticket] is written
};

// What one step reads besides the descriptor.
struct StepEnv {
    const uint8_t *arena;
    uint64_t block_size;
    uint64_t n_blocks;
    const SampleState *sample_st;
    const __half *q_buffer;
    float *o_buffer;
    uint32_t io_slots;
};

struct DwArgs {
    StepEnv env;
    CommandRing *ring;
    CompletionRing *comp;
    unsigned long long *step_count;
    uint32_t stop_sentinels;
    uint64_t idle_ns;
    DwCtl *ctl;
    DwQueue *queue;
};

struct DescF {
    uint64_t seq_id, cookie;
    uint32_t kv_block, out_offset, num_kv_blocks;
};

__device__ __forceinline__ DescF unpack_desc(uint4 a, uint4 b)
{
    DescF f;
    f.seq_id = (uint64_t)a.x | ((uint64_t)a.y << 32);
    f.kv_block = a.z;
    f.num_kv_blocks = a.w & 0xFFFFu;
    f.out_offset = b.x;
    f.cookie = (uint64_t)b.y | ((uint64_t)b.z << 32);
    return f;
}

__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t *p)
{
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ uint32_t ld_relaxed_gpu(const uint32_t *p)
{
    uint32_t v;
    asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void st_release_gpu(uint32_t *p, uint32_t v)
{
    asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Ring records live in pinned host memory shared with the CPU:
// system-scope relaxed 16-byte accesses (never served from a stale L1
// line, and free to be in flight together); ordering comes from the
// acquire of prod.tail / cons.head and the release of the indices.
__device__ __forceinline__ uint4 ld_relaxed_sys_v4(const void *p)
{
    uint4 r;
    asm volatile("ld.relaxed.sys.global.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p)
                 : "memory");
    return r;
}

__device__ __forceinline__ void st_relaxed_sys_v4(void *p, uint4 v)
{
    asm volatile("st.relaxed.sys.global.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x),
                 "r"(v.y), "r"(v.z), "r"(v.w)
                 : "memory");
}

// Plain (non-multicast) bulk copy global -> this CTA's shared memory,
// completion counted on an mbarrier in transaction bytes.  Both addresses
// 16-byte aligned, size a multiple of 16.
__device__ __forceinline__ void bulk_load(uint32_t dst, const void *src, uint32_t bytes,
                                          uint32_t bar)
{
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            dst),
        "l"(src), "r"(bytes), "r"(bar)
        : "memory");
}

__device__ __forceinline__ void set_error(DwCtl *ctl, int32_t code)
{
    if (ctl)
        atomicCAS(&ctl->error, 0, code);
}

// reference cu/attention_decode.cu:16-28
__device__ __forceinline__ float synth_query(const DescF &f, const SampleState *ss, uint32_t idx)
{
    uint64_t seed = f.seq_id ^ f.cookie ^ ((uint64_t)(idx + 1u) * 0x9e3779b97f4a7c15ull);
    if (ss)
        seed ^= *((const volatile uint64_t *)&ss->rng_state[idx & 3u]);
    const uint32_t bits = (uint32_t)(seed ^ (seed >> 32));
    const int centered = (int)(bits & 0xFFu) - 127;
    return (float)centered / 127.0f;
}

__device__ __forceinline__ void h8_to_f(uint4 v, float (&x)[8])
{
    const __half2 *h = reinterpret_cast<const __half2 *>(&v);
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const float2 f = __half22float2(h[i]);
        x[2 * i] = f.x;
        x[2 * i + 1] = f.y;
    }
}

enum StepStatus : uint32_t { kStepOk = 0, kStepBadBlock = 1, kStepCopyTimeout = 2 };

struct StepResult {
    uint32_t token, seq_len, status;
};

// One fixed128 decode step for descriptor f by the calling warp.  `stage`
// is the warp's shared-memory stage (KV rows, q, mbarrier), `phase` the
// parity of the stage's next mbarrier completion.  Uniform over the warp.
__device__ StepResult fixed128_step(const StepEnv &env, const DescF &f, uint8_t *stage,
                                    uint32_t &phase, uint32_t lane)
{
    StepResult r;
    // reference cu/worker.cu:39 (the step's seq_len is num_kv_blocks) and
    // cu/attention_decode.cu:76-78 (clamped to the 32-token block)
    uint32_t seq_len = f.num_kv_blocks == 0u ? 1u : f.num_kv_blocks;
    if (seq_len > KV_LAYOUT_TOKENS_PER_BLOCK)
        seq_len = KV_LAYOUT_TOKENS_PER_BLOCK;
    r.seq_len = seq_len;
    r.token = 0xFFFFFFFFu;
    if ((uint64_t)f.kv_block >= env.n_blocks) {
        r.status = kStepBadBlock;
        return r;
    }
    const uint32_t kv_s = rt::smem_u32(stage);
    const uint32_t bar = kv_s + kKvBytes + 512u;
    float *q_s = reinterpret_cast<float *>(stage + kKvBytes);
    const uint8_t *blk = env.arena + (uint64_t)f.kv_block * env.block_size;
    const uint32_t bytes = seq_len * kRowBytes;
    if (lane == 0) {
        // this warp's earlier generic reads of the stage precede the copy
        rt::fence_proxy_async_smem();
        rt::mbar_arrive_expect_tx(bar, 2u * bytes);
        bulk_load(kv_s, blk, bytes, bar);
        bulk_load(kv_s + kVPlane, blk + kVPlane, bytes, bar);
    }
    // the query while the rows are in flight (reference
    // cu/attention_decode.cu:30-46, cu/worker.cu:34-37)
    const uint32_t slot = env.io_slots == 0u ? 0u : (f.out_offset & (env.io_slots - 1u));
    float q4[4];
    if (env.q_buffer) {
        const uint2 raw = __ldcg(reinterpret_cast<const uint2 *>(env.q_buffer +
                                                                 (uint64_t)slot * 128u) + lane);
        const float2 a = __half22float2(*reinterpret_cast<const __half2 *>(&raw.x));
        const float2 b = __half22float2(*reinterpret_cast<const __half2 *>(&raw.y));
        q4[0] = a.x, q4[1] = a.y, q4[2] = b.x, q4[3] = b.y;
    } else {
#pragma unroll
        for (int j = 0; j < 4; j++)
            q4[j] = synth_query(f, env.sample_st, 4u * lane + j);
    }
    reinterpret_cast<float4 *>(q_s)[lane] = make_float4(q4[0], q4[1], q4[2], q4[3]);
    __syncwarp();
    bool ok = rt::mbar_wait_bounded(bar, phase, kCopyLimitNs);
    ok = __all_sync(0xFFFFFFFFu, ok);
    phase ^= 1u;
    if (!ok) {
        // the copy may still land: wait for it (bounded again) before the
        // stage is reused or the CTA exits
        rt::mbar_wait_bounded(bar, phase ^ 1u, kCopyLimitNs);
        r.status = kStepCopyTimeout;
        return r;
    }

    // score of token `lane`: eight ascending-d fma chains, d = i (mod 8)
    const float scale = rsqrtf((float)DECODE_FIXED_HEAD_DIM);
    float s = 0.0f;
    if (lane < seq_len) {  // lanes past seq_len would read rows that were not copied
        const uint8_t *krow = stage + lane * kRowBytes;
        float p[8];
#pragma unroll
        for (int i = 0; i < 8; i++)
            p[i] = 0.0f;
#pragma unroll 4
        for (uint32_t c = 0; c < 16u; c++) {
            float k[8];
            h8_to_f(*reinterpret_cast<const uint4 *>(krow + c * 16u), k);
            const float4 qa = reinterpret_cast<const float4 *>(q_s)[2u * c];
            const float4 qb = reinterpret_cast<const float4 *>(q_s)[2u * c + 1u];
            p[0] = __fmaf_rn(qa.x, k[0], p[0]);
            p[1] = __fmaf_rn(qa.y, k[1], p[1]);
            p[2] = __fmaf_rn(qa.z, k[2], p[2]);
            p[3] = __fmaf_rn(qa.w, k[3], p[3]);
            p[4] = __fmaf_rn(qb.x, k[4], p[4]);
            p[5] = __fmaf_rn(qb.y, k[5], p[5]);
            p[6] = __fmaf_rn(qb.z, k[6], p[6]);
            p[7] = __fmaf_rn(qb.w, k[7], p[7]);
        }
        s = (((p[0] + p[4]) + (p[2] + p[6])) + ((p[1] + p[5]) + (p[3] + p[7]))) * scale;
    }

    // online softmax over 16-token tiles; lane owns d = 4*lane .. 4*lane+3
    float o[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    float run_max = -INFINITY, run_norm = 0.0f;
    const uint8_t *vbase = stage + kVPlane + lane * 8u;
    for (uint32_t base = 0; base < seq_len; base += DECODE_TILE_TOKENS) {
        const uint32_t cnt = min(DECODE_TILE_TOKENS, seq_len - base);
        const bool mine = lane >= base && lane < base + cnt;
        float tmax = mine ? s : -INFINITY;
#pragma unroll
        for (int off = 16; off > 0; off >>= 1)
            tmax = fmaxf(tmax, __shfl_xor_sync(0xFFFFFFFFu, tmax, off));
        const float new_max = fmaxf(run_max, tmax);
        const float rescale = run_norm == 0.0f ? 0.0f : expf(run_max - new_max);
        const float e = expf(s - new_max);  // used for this tile's lanes only
        float tnorm = 0.0f;
        float acc[4];
#pragma unroll
        for (int j = 0; j < 4; j++)
            acc[j] = o[j] * rescale;
        for (uint32_t t = 0; t < cnt; t++) {
            const float w = __shfl_sync(0xFFFFFFFFu, e, base + t);
            tnorm += w;
            const uint2 vv = *reinterpret_cast<const uint2 *>(vbase + (base + t) * kRowBytes);
            const float2 v01 = __half22float2(*reinterpret_cast<const __half2 *>(&vv.x));
            const float2 v23 = __half22float2(*reinterpret_cast<const __half2 *>(&vv.y));
            acc[0] = __fmaf_rn(w, v01.x, acc[0]);
            acc[1] = __fmaf_rn(w, v01.y, acc[1]);
            acc[2] = __fmaf_rn(w, v23.x, acc[2]);
            acc[3] = __fmaf_rn(w, v23.y, acc[3]);
        }
#pragma unroll
        for (int j = 0; j < 4; j++)
            o[j] = acc[j];
        run_norm = __fmaf_rn(run_norm, rescale, tnorm);
        run_max = new_max;
    }
    if (run_norm == 0.0f)
        run_norm = 1.0f;
#pragma unroll
    for (int j = 0; j < 4; j++)
        o[j] = o[j] / run_norm;
    if (env.o_buffer)
        reinterpret_cast<float4 *>(env.o_buffer + (uint64_t)slot * 128u)[lane] =
            make_float4(o[0], o[1], o[2], o[3]);

    // argmax; rank = (d mod 32) * 4 + d / 32 orders ties as the reference
    // (cu/attention_decode.cu:171-194); only values above -inf count, none -> 0
    float bv = -INFINITY;
    uint32_t br = 0xFFFFFFFFu;
#pragma unroll
    for (int j = 0; j < 4; j++) {
        const uint32_t d = 4u * lane + j;
        const uint32_t rank = (d & 31u) * 4u + (d >> 5);
        if (o[j] > bv || (o[j] == bv && o[j] > -INFINITY && rank < br)) {
            bv = o[j];
            br = rank;
        }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        const float ov = __shfl_xor_sync(0xFFFFFFFFu, bv, off);
        const uint32_t orank = __shfl_xor_sync(0xFFFFFFFFu, br, off);
        if (ov > bv || (ov == bv && orank < br)) {
            bv = ov;
            br = orank;
        }
    }
    r.token = bv > -INFINITY ? (br & 3u) * 32u + (br >> 2) : 0u;
    r.status = kStepOk;
    __syncwarp();  // all lanes are done with the stage before it is refilled
    return r;
}

// reference cu/attention_decode.cu:196-203
__device__ __forceinline__ uint64_t cycle_estimate(uint32_t seq_len)
{
    const uint64_t tiles = (seq_len + DECODE_TILE_TOKENS - 1u) / DECODE_TILE_TOKENS;
    return tiles * (uint64_t)DECODE_FIXED_HEAD_DIM * 24ull;
}

__device__ void init_stage_barrier(uint8_t *stage, uint32_t lane)
{
    if (lane == 0) {
        rt::mbar_init(rt::smem_u32(stage) + kKvBytes + 512u, 1u);
        rt::mbar_fence_init();
    }
    __syncwarp();
}

// ---------------------------------------------------------------- pump
// Bits 0, 2, 4, ... 30 of x packed into bits 0..15.
__device__ __forceinline__ uint32_t even_bits(uint32_t x)
{
    x &= 0x55555555u;
    x = (x | (x >> 1)) & 0x33333333u;
    x = (x | (x >> 2)) & 0x0F0F0F0Fu;
    x = (x | (x >> 4)) & 0x00FF00FFu;
    return (x | (x >> 8)) & 0x0000FFFFu;
}

constexpr uint32_t kPieces = kPumpBatch * 2u / 32u;  // 16-byte ring pieces per lane per batch

__device__ void pump_loop(const DwArgs &a, uint32_t lane)
{
    DwCtl *ctl = a.ctl;
    DwQueue *qu = a.queue;
    uint32_t head = 0, ctail = 0, chead = 0;
    if (lane == 0) {
        head = rt_load_relaxed_u32(&a.ring->cons.head);
        ctail = rt_load_relaxed_u32(&a.comp->prod.tail);
        chead = rt_load_acquire_u32(&a.comp->cons.head);
        ctl->workers = gridDim.x * kWarpsPerCta - 1u;
    }
    head = __shfl_sync(0xFFFFFFFFu, head, 0);
    ctail = __shfl_sync(0xFFFFFFFFu, ctail, 0);
    chead = __shfl_sync(0xFFFFFFFFu, chead, 0);
    __syncwarp();  // every lane's ring accesses after lane 0's acquire
    uint32_t tail_seen = head;  // last prod.tail observed: records below it are published
    uint32_t published = 0, drained = 0, sentinels = 0;
    unsigned long long consumed = 0;
    bool consuming = true, full_noted = false;
    int32_t err = 0;
    uint32_t nap = 32;
    uint64_t t_last = rt::globaltimer_ns();

    while (true) {
        bool progress = false;

        // 1. issue this pass's ring reads; they complete while the drain runs.
        //    Instruction j, lane l reads 16-byte piece 32j + l of the batch
        //    (half l & 1 of record 16j + l / 2): 512 contiguous bytes per
        //    instruction, whole lines over the host link.
        uint32_t n = 0;
        uint4 piece[kPieces];
        if (consuming) {
            if (tail_seen - head < kPumpBatch) {  // the cached tail cannot fill a batch
                uint32_t t = 0;
                if (lane == 0)
                    t = rt_load_acquire_u32(&a.ring->prod.tail);
                tail_seen = __shfl_sync(0xFFFFFFFFu, t, 0);
                // __shfl_sync moves the value but orders no memory; the warp
                // barrier puts every lane's record loads below after lane 0's
                // acquire of the tail.
                __syncwarp();
            }
            const uint32_t avail = tail_seen - head;
            if (avail > (uint32_t)RING_SIZE) {  // the host broke the ring contract
                err = RT_EDEVICE;
                break;
            }
            n = min(min(avail, kQueue - (published - drained)), kPumpBatch);
#pragma unroll
            for (uint32_t j = 0; j < kPieces; j++) {
                const uint32_t r = 16u * j + (lane >> 1);
                piece[j] = make_uint4(0, 0, 0, 0);
                if (r < n)
                    piece[j] = ld_relaxed_sys_v4(
                        reinterpret_cast<const uint8_t *>(
                            &a.ring->slots[(head + r) & (RING_SIZE - 1u)]) + 16u * (lane & 1u));
            }
        }

        // 2. deliver finished completions in ticket (= ring) order: a batch's
        //    ready words and records are read with all loads in flight, then
        //    written to the CompletionRing with one tail release
        bool ring_full = false;
        if (drained != published) {
            const uint32_t look = min(published - drained, kPumpBatch);
            uint32_t rbits = 0;
#pragma unroll
            for (uint32_t j = 0; j < kPumpBatch / 32u; j++) {
                const uint32_t e = 32u * j + lane;
                if (e < look &&
                    ld_relaxed_gpu(&qu->ready[(drained + e) & (kQueue - 1u)]) == drained + e + 1u)
                    rbits |= 1u << j;
            }
            uint32_t k = 0;
#pragma unroll
            for (uint32_t j = 0; j < kPumpBatch / 32u; j++) {
                const uint32_t m = __ballot_sync(0xFFFFFFFFu, (rbits >> j) & 1u);
                const uint32_t t = m == 0xFFFFFFFFu ? 32u : (uint32_t)(__ffs(~m) - 1);
                k += t;
                if (t < 32u)
                    break;
            }
            if (k) {
                __threadfence();  // the ready words observed before the records are read
                uint32_t room = (uint32_t)COMP_RING_SIZE - (ctail - chead);
                if (room < k) {
                    if (lane == 0)
                        chead = rt_load_acquire_u32(&a.comp->cons.head);
                    chead = __shfl_sync(0xFFFFFFFFu, chead, 0);
                    __syncwarp();  // slot stores below after lane 0's acquire
                    room = (uint32_t)COMP_RING_SIZE - (ctail - chead);
                }
                ring_full = room < k;
                k = min(k, room);
            }
            if (k) {
                uint4 c[kPumpBatch / 16u];
#pragma unroll
                for (uint32_t j = 0; j < kPumpBatch / 16u; j++) {
                    // piece e = 32j + lane: half (e & 1) of entry e / 2
                    const uint32_t e = (32u * j + lane) >> 1;
                    c[j] = make_uint4(0, 0, 0, 0);
                    if (e < k)
                        c[j] = __ldcg(&qu->comp[2u * ((drained + e) & (kQueue - 1u)) + (lane & 1u)]);
                }
#pragma unroll
                for (uint32_t j = 0; j < kPumpBatch / 16u; j++) {
                    const uint32_t e = (32u * j + lane) >> 1;
                    if (e < k)
                        st_relaxed_sys_v4(reinterpret_cast<uint8_t *>(
                                              &a.comp->slots[(ctail + e) & (COMP_RING_SIZE - 1u)]) +
                                              16u * (lane & 1u),
                                          c[j]);
                }
                __syncwarp();
                __threadfence_system();
                if (lane == 0) {
                    rt_store_release_u32(&a.comp->prod.tail, ctail + k);
                    if (a.step_count)
                        atomicAdd(a.step_count, (unsigned long long)k);
                    st_release_gpu(&ctl->drained.v, drained + k);
                }
                ctail += k;
                drained += k;
                progress = true;
                full_noted = false;
            }
        }
        if (ring_full) {
            // one count per stall (the reference counts every retry)
            if (!full_noted && lane == 0) {
                comp_ring_record_overflow(&a.comp->overflow.value);
                ctl->comp_full++;
            }
            full_noted = true;
        }

        // 3. take the ring records read in step 1: compact the work into the
        //    queue, stop after the stop_sentinels-th sentinel
        if (n) {
            uint32_t taken = 0;
            const uint32_t m = lane >> 1;  // record of this lane within an instruction
#pragma unroll
            for (uint32_t j = 0; j < kPieces; j++) {
                const uint32_t rb = 16u * j;
                if (rb >= n || !consuming)
                    break;
                const bool valid = rb + m < n;
                const bool even = (lane & 1u) == 0u;
                const uint32_t smask = even_bits(__ballot_sync(
                    0xFFFFFFFFu, even && valid && piece[j].x == 0xFFFFFFFFu &&
                                     piece[j].y == 0xFFFFFFFFu));
                uint32_t take = even_bits(__ballot_sync(0xFFFFFFFFu, even && valid));
                const uint32_t need = a.stop_sentinels - sentinels;
                if ((uint32_t)__popc(smask) >= need) {
                    // cut right after the need-th sentinel of this group
                    uint32_t mm = smask;
                    for (uint32_t q = 1; q < need; q++)
                        mm &= mm - 1u;
                    const uint32_t last = __ffs(mm) - 1u;
                    take &= (2u << last) - 1u;
                    consuming = false;
                }
                const uint32_t work = take & ~smask;
                if ((work >> m) & 1u) {
                    const uint32_t qi = (published + __popc(work & ((1u << m) - 1u))) & (kQueue - 1u);
                    qu->desc[2u * qi + (lane & 1u)] = piece[j];
                }
                published += __popc(work);
                sentinels += __popc(take & smask);
                taken += __popc(take);
            }
            if (taken) {
                __syncwarp();
                __threadfence();
                if (lane == 0) {
                    st_release_gpu(&ctl->published.v, published);
                    rt_store_release_u32(&a.ring->cons.head, head + taken);
                }
                head += taken;
                consumed += taken;
                progress = true;
            }
            if (!consuming && lane == 0)
                st_release_gpu(&ctl->stop.v, 1u);
        }

        if (!consuming && drained == published)
            break;
        uint64_t now = 0;
        if (lane == 0)
            now = rt::globaltimer_ns();
        now = __shfl_sync(0xFFFFFFFFu, now, 0);
        if (progress) {
            t_last = now;
            nap = 32;
        } else {
            if (now - t_last > a.idle_ns) {
                err = RT_ETIMEOUT;
                break;
            }
            __nanosleep(nap);
            nap = min(nap * 2u, 256u);
        }
    }
    if (lane == 0) {
        if (err)
            set_error(ctl, err);
        st_release_gpu(&ctl->stop.v, 1u);
        ctl->consumed = consumed;
        ctl->completed = drained;
        ctl->sentinels = sentinels;
        __threadfence();
        ctl->finished = 1u;
    }
}

// -------------------------------------------------------------- workers
__device__ void worker_loop(const DwArgs &a, uint8_t *stage, uint32_t lane)
{
    DwCtl *ctl = a.ctl;
    DwQueue *qu = a.queue;
    uint32_t phase = 0;
    const uint64_t limit = a.idle_ns + kWorkerMarginNs;
    while (true) {
        uint32_t t = 0;
        bool have = false;
        if (lane == 0) {
            t = atomicAdd(&ctl->claimed.v, 1u);
            uint32_t seen_p = 0xFFFFFFFFu, seen_d = 0xFFFFFFFFu, nap = 64;
            uint64_t t0 = 0;
            while (true) {
                uint32_t p = ld_acquire_gpu(&ctl->published.v);
                if ((int32_t)(p - t) > 0) {
                    have = true;
                    break;
                }
                if (ld_acquire_gpu(&ctl->stop.v)) {
                    p = ld_acquire_gpu(&ctl->published.v);
                    have = (int32_t)(p - t) > 0;
                    break;
                }
                // the clock restarts whenever the pump moves, so only a
                // pump that stopped making progress can run it out
                const uint32_t d = ld_relaxed_gpu(&ctl->drained.v);
                const uint64_t now = rt::globaltimer_ns();
                if (p != seen_p || d != seen_d) {
                    seen_p = p;
                    seen_d = d;
                    t0 = now;
                } else if (now - t0 > limit) {
                    set_error(ctl, RT_ETIMEOUT);
                    break;
                }
                __nanosleep(nap);
                nap = min(nap * 2u, 512u);
            }
        }
        have = __shfl_sync(0xFFFFFFFFu, have, 0);
        // orders the other lanes' queue reads after lane 0's acquire of
        // `published` (a shuffle alone orders no memory)
        __syncwarp();
        if (!have)
            break;
        t = __shfl_sync(0xFFFFFFFFu, t, 0);
        const uint32_t qi = t & (kQueue - 1u);
        const DescF f = unpack_desc(__ldcg(&qu->desc[2u * qi]), __ldcg(&qu->desc[2u * qi + 1u]));
        const StepResult r = fixed128_step(a.env, f, stage, phase, lane);
        if (lane == 0) {
            if (r.status == kStepBadBlock) {
                if (atomicCAS(&ctl->error, 0, RT_EDEVICE) == 0)
                    ctl->bad_block = f.kv_block;
            } else if (r.status == kStepCopyTimeout) {
                set_error(ctl, RT_ETIMEOUT);
            }
            const uint64_t cyc = r.status == kStepOk ? cycle_estimate(r.seq_len) : 0ull;
            // Completion {seq_id, token_id, kv_block_offset, reward_cookie,
            // cycles_taken} (reference cu/worker.cu:53-59)
            __stcg(&qu->comp[2u * qi], make_uint4((uint32_t)f.seq_id, (uint32_t)(f.seq_id >> 32),
                                                  r.token, f.kv_block));
            __stcg(&qu->comp[2u * qi + 1u], make_uint4((uint32_t)f.cookie,
                                                       (uint32_t)(f.cookie >> 32), (uint32_t)cyc,
                                                       (uint32_t)(cyc >> 32)));
            __threadfence();
            st_release_gpu(&qu->ready[qi], t + 1u);
        }
        if (r.status == kStepCopyTimeout)
            break;
    }
}

__global__ void __launch_bounds__(kWarpsPerCta * 32) decode_worker_kernel(DwArgs a)
{
    extern __shared__ __align__(128) uint8_t smem[];
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    uint8_t *stage = smem + warp * kStageBytes;
    if (blockIdx.x == 0 && warp == 0) {
        pump_loop(a, lane);
        return;
    }
    init_stage_barrier(stage, lane);
    worker_loop(a, stage, lane);
}

// Standalone step over a device array of descriptors: one warp each.
__global__ void __launch_bounds__(kWarpsPerCta * 32)
    fixed128_batch_kernel(StepEnv env, const uint4 *descs, uint32_t n, DecodeStepResult *out)
{
    extern __shared__ __align__(128) uint8_t smem[];
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    const uint32_t i = blockIdx.x * kWarpsPerCta + warp;
    if (i >= n)
        return;
    uint8_t *stage = smem + warp * kStageBytes;
    init_stage_barrier(stage, lane);
    uint32_t phase = 0;
    const DescF f = unpack_desc(descs[2u * i], descs[2u * i + 1u]);
    const StepResult r = fixed128_step(env, f, stage, phase, lane);
    if (lane == 0) {
        DecodeStepResult res;
        const bool ok = r.status == kStepOk;
        res.path_kind = ok ? DECODE_PATH_FIXED128 : DECODE_PATH_STUB;
        res.token_id = r.token;
        res.bytes_touched = ok ? r.seq_len * DECODE_FIXED_HEAD_DIM * KV_LAYOUT_SCALAR_BYTES * 2u : 0u;
        res.tile_count = ok ? (r.seq_len + DECODE_TILE_TOKENS - 1u) / DECODE_TILE_TOKENS : 0u;
        res.cycle_estimate = ok ? cycle_estimate(r.seq_len) : 0ull;
        out[i] = res;
    }
}

// ------------------------------------------------------------------ host
std::mutex g_dw_mu;
DwCtl *g_dw_ctl[64] = {};
DwQueue *g_dw_queue[64] = {};
cudaEvent_t g_dw_done[64] = {};

int fill_env(const KVArena *arena, const SampleState *sample_st, const void *q_buffer,
             float *o_buffer, uint32_t io_slots, StepEnv *env, const char *what)
{
    if (!arena || !arena->base || arena->block_size < kKvBytes || arena->block_size % 16u ||
        (uintptr_t)arena->base % 16u) {
        rt::set_error("%s: the arena needs a device base and blocks of >= %u bytes, 16-byte "
                      "aligned", what, kKvBytes);
        return RT_EINVAL;
    }
    if (((uintptr_t)q_buffer % 16u) || ((uintptr_t)o_buffer % 16u)) {
        rt::set_error("%s: q_buffer and o_buffer must be 16-byte aligned", what);
        return RT_EINVAL;
    }
    env->arena = arena->base;
    env->block_size = arena->block_size;
    env->n_blocks = arena->capacity / arena->block_size;
    env->sample_st = sample_st;
    env->q_buffer = static_cast<const __half *>(q_buffer);
    env->o_buffer = o_buffer;
    env->io_slots = io_slots;
    return RT_OK;
}

template <typename K>
cudaError_t allow_smem(K kernel)
{
    return cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)(kWarpsPerCta * kStageBytes));
}

// Pinned host rings are device-mapped; translate in case the device
// address differs from the host address.
template <typename T>
T *mapped(T *p)
{
    void *d = nullptr;
    if (cudaHostGetDevicePointer(&d, (void *)p, 0) == cudaSuccess && d)
        return static_cast<T *>(d);
    (void)cudaGetLastError();
    return p;
}

}  // namespace

extern "C" int rt_attention_fixed128(const Descriptor *descs, uint32_t n, const KVArena *arena,
                                     const SampleState *sample_st, const void *q_buffer,
                                     float *o_buffer, uint32_t io_slots,
                                     DecodeStepResult *results, void *stream)
{
    StepEnv env;
    int rc = fill_env(arena, sample_st, q_buffer, o_buffer, io_slots, &env, "attention_fixed128");
    if (rc != RT_OK)
        return rc;
    if (n == 0u)
        return RT_OK;
    if (!descs || !results || ((uintptr_t)descs % 16u) || ((uintptr_t)results % 8u)) {
        rt::set_error("attention_fixed128: descs (16-byte aligned) and results are required");
        return RT_EINVAL;
    }
    cudaError_t err = allow_smem(fixed128_batch_kernel);
    if (err != cudaSuccess)
        return rt::cuda_fail(err, "attention_fixed128: smem attribute");
    const uint32_t grid = (n + kWarpsPerCta - 1u) / kWarpsPerCta;
    fixed128_batch_kernel<<<grid, kWarpsPerCta * 32, kWarpsPerCta * kStageBytes,
                            (cudaStream_t)stream>>>(env, reinterpret_cast<const uint4 *>(descs), n,
                                                    results);
    err = cudaGetLastError();
    return err == cudaSuccess ? RT_OK : rt::cuda_fail(err, "attention_fixed128: launch");
}

extern "C" int rt_launch_decode_worker(CommandRing *ring, const KVArena *arena,
                                       CompletionRing *comp_ring, const SampleState *sample_st,
                                       const void *q_buffer, float *o_buffer, uint32_t io_slots,
                                       uint64_t *step_count, uint32_t stop_sentinels,
                                       uint32_t idle_timeout_ms, void *stream)
{
    if (!ring || !comp_ring) {
        rt::set_error("decode_worker: null ring");
        return RT_EINVAL;
    }
    DwArgs a;
    memset(&a, 0, sizeof(a));
    int rc = fill_env(arena, sample_st, q_buffer, o_buffer, io_slots, &a.env, "decode_worker");
    if (rc != RT_OK)
        return rc;
    int dev = 0;
    cudaError_t err = cudaGetDevice(&dev);
    if (err != cudaSuccess)
        return rt::cuda_fail(err, "decode_worker: device");
    if (dev < 0 || dev >= 64) {
        rt::set_error("decode_worker: device index %d out of range", dev);
        return RT_EINVAL;
    }
    int sms = 0;
    err = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (err != cudaSuccess)
        return rt::cuda_fail(err, "decode_worker: SM count");
    cudaStream_t s = (cudaStream_t)stream;
    std::lock_guard<std::mutex> lk(g_dw_mu);
    if (!g_dw_ctl[dev]) {
        err = cudaMalloc(&g_dw_ctl[dev], sizeof(DwCtl));
        if (err == cudaSuccess)
            err = cudaMalloc(&g_dw_queue[dev], sizeof(DwQueue));
        if (err == cudaSuccess)
            err = cudaEventCreateWithFlags(&g_dw_done[dev], cudaEventDisableTiming);
        if (err != cudaSuccess)
            return rt::cuda_fail(err, "decode_worker: control block");
    } else {
        err = cudaEventQuery(g_dw_done[dev]);
        if (err == cudaErrorNotReady) {
            (void)cudaGetLastError();
            rt::set_error("decode_worker: a decode worker is still running on device %d", dev);
            return RT_EINVAL;
        }
        if (err != cudaSuccess)
            return rt::cuda_fail(err, "decode_worker: previous launch");
    }
    err = allow_smem(decode_worker_kernel);
    if (err != cudaSuccess)
        return rt::cuda_fail(err, "decode_worker: smem attribute");
    int per_sm = 0;
    err = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, decode_worker_kernel,
                                                        kWarpsPerCta * 32,
                                                        kWarpsPerCta * kStageBytes);
    if (err != cudaSuccess || per_sm < 1)
        return rt::cuda_fail(err != cudaSuccess ? err : cudaErrorInvalidConfiguration,
                             "decode_worker: occupancy");
    // one CTA per SM: every CTA is resident, so no worker waits on a CTA
    // that cannot start
    const uint32_t grid = (uint32_t)sms;
    a.ring = mapped(ring);
    a.comp = mapped(comp_ring);
    a.step_count = reinterpret_cast<unsigned long long *>(step_count);
    a.stop_sentinels = stop_sentinels ? stop_sentinels : (uint32_t)sms;
    a.idle_ns = (uint64_t)(idle_timeout_ms ? idle_timeout_ms : 10000u) * 1000000ull;
    a.ctl = g_dw_ctl[dev];
    a.queue = g_dw_queue[dev];
    // stream-ordered resets (no host synchronisation): the control block
    // (the pump fills in the worker count) and the ready words
    err = cudaMemsetAsync(a.ctl, 0, sizeof(DwCtl), s);
    if (err == cudaSuccess)
        err = cudaMemsetAsync(a.queue->ready, 0, sizeof(a.queue->ready), s);
    if (err != cudaSuccess)
        return rt::cuda_fail(err, "decode_worker: setup");
    decode_worker_kernel<<<grid, kWarpsPerCta * 32, kWarpsPerCta * kStageBytes, s>>>(a);
    err = cudaGetLastError();
    if (err != cudaSuccess)
        return rt::cuda_fail(err, "decode_worker: launch");
    err = cudaEventRecord(g_dw_done[dev], s);
    return err == cudaSuccess ? RT_OK : rt::cuda_fail(err, "decode_worker: event");
}

extern "C" int rt_decode_worker_stats(void *stream, rt_decode_worker_stats_t *st)
{
    int dev = 0;
    cudaGetDevice(&dev);
    if (!st || dev < 0 || dev >= 64 || !g_dw_ctl[dev]) {
        rt::set_error("decode_worker_stats: no decode worker was launched on this device");
        return RT_EINVAL;
    }
    DwCtl c;
    cudaError_t err = cudaMemcpyAsync(&c, g_dw_ctl[dev], sizeof(c), cudaMemcpyDeviceToHost,
                                      (cudaStream_t)stream);
    if (err == cudaSuccess)
        err = cudaStreamSynchronize((cudaStream_t)stream);
    if (err != cudaSuccess)
        return rt::cuda_fail(err, "decode_worker_stats");
    memset(st, 0, sizeof(*st));
    st->consumed = c.finished ? c.consumed : 0ull;
    st->completed = c.finished ? c.completed : (uint64_t)c.drained.v;
    st->published = c.published.v;
    st->sentinels = c.sentinels;
    st->comp_ring_full = c.comp_full;
    st->error = c.error;
    st->bad_block = c.bad_block;
    st->workers = c.workers;
    st->finished = c.finished;
    return RT_OK;
}
