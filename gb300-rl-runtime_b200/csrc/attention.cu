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
//    numbered sequence-fastest: sequences that share prefix pages (a GRPO
//    group) run side by side and the shared pages come from L2.
//  * Staging: per page the warp's elected lane issues four 2-D TMA tensor
//    loads (K and V, two 64-column halves each, 128-byte swizzle) into one
//    8 KiB stage of the warp's 3-stage ring, completion tracked by a
//    shared-memory mbarrier with transaction bytes (no multicast).
//  * Math: the G query heads of the KV group form the rows of one
//    m16n8k16 bf16 tensor-core tile (rows >= G are zero), so S = Q.K^T and
//    O += P.V are each 16 mma per page; the S accumulator layout is reused
//    directly as the A operand of P.V.  Softmax runs in registers in the log2
//    domain with quad shuffles for the row max.
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

constexpr int kWarps = 4;            // warps (independent items) per CTA
constexpr int kStages = 3;           // pipeline depth per warp
constexpr int kStageBytes = 8192;    // K (2 x 2 KiB halves) + V (2 x 2 KiB)
constexpr int kMaxChunkPages = 64;   // page ids live in two registers per lane
constexpr int kSmemBytes = kWarps * kStages * kStageBytes + 1024;  // + 1 KiB alignment slack
constexpr uint64_t kWaitLimitNs = 2000000000ull;                    // 2 s per pipeline wait

enum : int32_t { kErrSeqLen = 1, kErrPage = 2, kErrTimeout = 3 };

struct AttnArgs {
    const __nv_bfloat16 *q;
    const int32_t *page_table;
    const int32_t *seq_lens;
    float *out;
    float *part_o;      // [B][Hkv][max_chunks][G][128]
    float *part_ml;     // [B][Hkv][max_chunks][G][2]  (max, sum) in log2 domain
    int32_t *counters;  // [B][Hkv]
    int32_t *error;
    unsigned long long *work_next;  // item dispenser (dynamic scheduling)
    unsigned int *work_done;        // warps that left the loop
    uint32_t num_seqs, num_q_heads, num_kv_heads, max_pages, max_chunks, chunk_pages, max_seq_len;
    uint64_t arena_pages;
    uint64_t n_items;
    float scale_log2;
    uint32_t evict_first;
};

__device__ __forceinline__ void flag_error(int32_t *err, int32_t code)
{
    atomicCAS(err, 0, code);
}

// One warp processes one item; see the file comment.  Returns false when a
// pipeline wait expired (the warp then stops taking items).
template <int G>
__device__ __forceinline__ bool process_item(const CUtensorMap &kv_map, const AttnArgs &a,
                                             uint64_t item, uint32_t stage0, uint8_t *base_ptr,
                                             uint32_t base_u32, uint64_t (&bars)[kStages],
                                             uint32_t &phases, uint64_t policy)
{
    const int lane = threadIdx.x & 31;
    const uint32_t B = a.num_seqs, Hq = a.num_q_heads, Hkv = a.num_kv_heads;
    const uint32_t b = (uint32_t)(item % B);
    const uint64_t rest = item / B;
    const uint32_t h = (uint32_t)(rest % Hkv);
    const int chunk = (int)(rest / Hkv);
    const int L = a.seq_lens[b];

    if (L < 0 || (uint32_t)L > a.max_seq_len || (uint32_t)L > a.max_pages * 16u) {
        if (lane == 0 && chunk == 0)
            flag_error(a.error, kErrSeqLen);
        return true;
    }
    if (L == 0) {
        if (chunk == 0)
            for (int i = lane; i < G * 128; i += 32)
                a.out[((size_t)b * Hq + (size_t)h * G) * 128 + i] = 0.0f;
        return true;
    }
    const int n_pages = (L + 15) >> 4;
    const int cp = (int)a.chunk_pages;
    const int n_chunks = (n_pages + cp - 1) / cp;
    if (chunk >= n_chunks)
        return true;
    const int p_begin = chunk * cp;
    const int n_mine = min(n_pages, p_begin + cp) - p_begin;

    // Page ids of this item: lane i holds pages i and 32 + i.
    const int32_t *ptab = a.page_table + (size_t)b * a.max_pages + p_begin;
    int pg_lo = 0, pg_hi = 0;
    if (lane < n_mine)
        pg_lo = ptab[lane];
    if (lane + 32 < n_mine)
        pg_hi = ptab[lane + 32];
    const bool bad = (lane < n_mine && (pg_lo < 0 || (uint64_t)pg_lo >= a.arena_pages)) ||
                     (lane + 32 < n_mine && (pg_hi < 0 || (uint64_t)pg_hi >= a.arena_pages));
    if (bad) {
        flag_error(a.error, kErrPage);
        if (pg_lo < 0 || (uint64_t)pg_lo >= a.arena_pages)
            pg_lo = 0;
        if (pg_hi < 0 || (uint64_t)pg_hi >= a.arena_pages)
            pg_hi = 0;
    }

    auto issue = [&](int i, int s) {
        const int pg = __shfl_sync(0xffffffffu, i < 32 ? pg_lo : pg_hi, i & 31);
        if (lane == 0) {
            const uint32_t bar = rt::smem_u32(&bars[s]);
            const uint32_t dst = stage0 + (uint32_t)(s * kStageBytes);
            const int32_t row_k = (int32_t)(((int64_t)pg * Hkv + h) * 32);
            rt::mbar_arrive_expect_tx(bar, (uint32_t)kStageBytes);
            rt::tma_load_2d(dst, &kv_map, 0, row_k, bar, policy);
            rt::tma_load_2d(dst + 2048u, &kv_map, 64, row_k, bar, policy);
            rt::tma_load_2d(dst + 4096u, &kv_map, 0, row_k + 16, bar, policy);
            rt::tma_load_2d(dst + 6144u, &kv_map, 64, row_k + 16, bar, policy);
        }
    };
    // The stage ring was left idle by the previous item: order this warp's
    // earlier generic accesses of it before the new TMA writes.
    rt::fence_proxy_async_smem();
    for (int i = 0; i < n_mine && i < kStages; i++)
        issue(i, i);

    // Q fragment: row r = lane/4 is query head h*G + r (rows >= G are zero);
    // k-step j covers dims 16j..16j+15.
    const int r = lane >> 2, q4 = lane & 3;
    uint32_t qa[8][4];
    {
        const uint32_t *qrow = reinterpret_cast<const uint32_t *>(
            a.q + ((size_t)b * Hq + (size_t)h * G + (r < G ? r : 0)) * 128);
#pragma unroll
        for (int j = 0; j < 8; j++) {
            qa[j][0] = r < G ? qrow[8 * j + q4] : 0u;
            qa[j][2] = r < G ? qrow[8 * j + 4 + q4] : 0u;
            qa[j][1] = 0u;
            qa[j][3] = 0u;
        }
    }

    float o[16][4];
#pragma unroll
    for (int n = 0; n < 16; n++)
        o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.0f;
    float m_run = -INFINITY, l_run = 0.0f;

    // Per-lane ldmatrix row offsets (swizzled chunk index = chunk ^ row%8).
    const int mi = lane >> 3, rr = lane & 7;
    const uint32_t k_row = (uint32_t)((((mi >> 1) << 3) + rr) * 128);
    const uint32_t v_row = (uint32_t)((((mi & 1) << 3) + rr) * 128);

    for (int i = 0; i < n_mine; i++) {
        const int s = i % kStages;
        const bool ok = rt::mbar_wait_bounded(rt::smem_u32(&bars[s]), (phases >> s) & 1u,
                                              kWaitLimitNs);
        if (!__all_sync(0xffffffffu, ok)) {
            if (lane == 0)
                flag_error(a.error, kErrTimeout);
            // Give copies still in flight a bounded chance to land before the
            // shared memory is released.
            for (int s2 = 0; s2 < kStages; s2++)
                (void)rt::mbar_wait_bounded(rt::smem_u32(&bars[s2]), (phases >> s2) & 1u,
                                            kWaitLimitNs / 4);
            return false;
        }
        phases ^= 1u << s;
        const uint32_t st = stage0 + (uint32_t)(s * kStageBytes);
        const int valid = min(16, L - (p_begin + i) * 16);
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

        // S = Q K^T for 16 tokens (two n-tiles of 8).
        float sc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
        for (int j = 0; j < 8; j++) {
            const int c = ((j & 3) << 1) + (mi & 1);
            const uint32_t addr = st + (uint32_t)((j >> 2) * 2048) + k_row + (uint32_t)((c ^ rr) << 4);
            uint32_t k0, k1, k2, k3;
            rt::ldsm_x4(addr, k0, k1, k2, k3);
            rt::mma_bf16_16816(sc[0], qa[j], k0, k1);
            rt::mma_bf16_16816(sc[1], qa[j], k2, k3);
        }

        float x0 = sc[0][0] * a.scale_log2, x1 = sc[0][1] * a.scale_log2;
        float x2 = sc[1][0] * a.scale_log2, x3 = sc[1][1] * a.scale_log2;
        if (valid < 16) {
            const int t0 = 2 * q4;
            if (t0 >= valid) x0 = -INFINITY;
            if (t0 + 1 >= valid) x1 = -INFINITY;
            if (t0 + 8 >= valid) x2 = -INFINITY;
            if (t0 + 9 >= valid) x3 = -INFINITY;
        }
        float mx = fmaxf(fmaxf(x0, x1), fmaxf(x2, x3));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
        const float m_new = fmaxf(m_run, mx);
        const float corr = rt::fast_exp2(m_run - m_new);
        const float p0 = rt::fast_exp2(x0 - m_new), p1 = rt::fast_exp2(x1 - m_new);
        const float p2 = rt::fast_exp2(x2 - m_new), p3 = rt::fast_exp2(x3 - m_new);
        l_run = l_run * corr + ((p0 + p1) + (p2 + p3));
        m_run = m_new;
#pragma unroll
        for (int n = 0; n < 16; n++) {
            o[n][0] *= corr;
            o[n][1] *= corr;
        }
        const uint32_t pa[4] = {rt::pack_bf16x2(p0, p1), 0u, rt::pack_bf16x2(p2, p3), 0u};

        // O += P V over 128 dims (16 n-tiles of 8, two per ldmatrix.x4).
#pragma unroll
        for (int dd = 0; dd < 8; dd++) {
            const int c = ((dd & 3) << 1) + (mi >> 1);
            const uint32_t addr =
                st + 4096u + (uint32_t)((dd >> 2) * 2048) + v_row + (uint32_t)((c ^ rr) << 4);
            uint32_t v0, v1, v2, v3;
            rt::ldsm_x4_trans(addr, v0, v1, v2, v3);
            rt::mma_bf16_16816(o[2 * dd], pa, v0, v1);
            rt::mma_bf16_16816(o[2 * dd + 1], pa, v2, v3);
        }
        __syncwarp();
        if (i + kStages < n_mine) {
            // The stage's shared memory was only read (ldmatrix, consumed by
            // the mma above) unless this was a tail page whose V rows were
            // zeroed: only generic writes need ordering before the TMA write.
            if (valid < 16)
                rt::fence_proxy_async_smem();
            issue(i + kStages, s);
        }
    }
    l_run += __shfl_xor_sync(0xffffffffu, l_run, 1);
    l_run += __shfl_xor_sync(0xffffffffu, l_run, 2);

    const size_t bh = (size_t)b * Hkv + h;
    if (n_chunks == 1) {
        if (r < G) {
            const float inv = 1.0f / l_run;
            float *dst = a.out + ((size_t)b * Hq + (size_t)h * G + r) * 128 + 2 * q4;
#pragma unroll
            for (int n = 0; n < 16; n++)
                *reinterpret_cast<float2 *>(dst + n * 8) = make_float2(o[n][0] * inv, o[n][1] * inv);
        }
        return true;
    }

    // ---- split-K: write this chunk's partial; the last warp merges ----
    if (r < G) {
        const size_t pi = (bh * a.max_chunks + chunk) * G + r;
        float *dst = a.part_o + pi * 128 + 2 * q4;
#pragma unroll
        for (int n = 0; n < 16; n++)
            *reinterpret_cast<float2 *>(dst + n * 8) = make_float2(o[n][0], o[n][1]);
        if (q4 == 0)
            *reinterpret_cast<float2 *>(a.part_ml + pi * 2) = make_float2(m_run, l_run);
    }
    __threadfence();
    __syncwarp();
    int prev = 0;
    if (lane == 0)
        prev = atomicAdd(&a.counters[bh], 1);
    prev = __shfl_sync(0xffffffffu, prev, 0);
    if (prev != n_chunks - 1)
        return true;
    __threadfence();
    for (int row = 0; row < G; row++) {
        float M = -INFINITY;
        for (int c = 0; c < n_chunks; c++)
            M = fmaxf(M, __ldcg(&a.part_ml[((bh * a.max_chunks + c) * G + row) * 2]));
        float Ls = 0.0f;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int c = 0; c < n_chunks; c++) {
            const size_t pi = (bh * a.max_chunks + c) * G + row;
            const float2 ml = __ldcg(reinterpret_cast<const float2 *>(&a.part_ml[pi * 2]));
            const float wt = rt::fast_exp2(ml.x - M);
            Ls += ml.y * wt;
            const float4 v = __ldcg(reinterpret_cast<const float4 *>(&a.part_o[pi * 128 + lane * 4]));
            acc.x += v.x * wt;
            acc.y += v.y * wt;
            acc.z += v.z * wt;
            acc.w += v.w * wt;
        }
        const float inv = 1.0f / Ls;
        *reinterpret_cast<float4 *>(a.out + ((size_t)b * Hq + (size_t)h * G + row) * 128 + lane * 4) =
            make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv);
    }
    if (lane == 0)
        a.counters[bh] = 0;
    return true;
}

// Persistent warps take items in increasing order from a global dispenser
// (one atomic per item, fetched one item ahead), so a warp whose item is
// empty moves on at once, long and short items balance dynamically, and the
// items of a GRPO group's sequences run side by side.  The last warp to
// leave resets the dispenser for the next launch.
template <int G>
__global__ void __launch_bounds__(kWarps * 32, 2)
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

    if (lane == 0) {
        rt::prefetch_tensormap(&kv_map);
        for (int s = 0; s < kStages; s++)
            rt::mbar_init(rt::smem_u32(&bars[warp][s]), 1u);
        rt::mbar_fence_init();
        rt::fence_proxy_async_smem();
    }
    __syncwarp();
    const uint64_t policy = a.evict_first ? rt::l2_policy_evict_first() : rt::l2_policy_evict_normal();
    uint32_t phases = 0;
    unsigned long long grab = 0;
    if (lane == 0)
        grab = atomicAdd(a.work_next, 1ull);
    uint64_t item = __shfl_sync(0xffffffffu, grab, 0);
    while (item < a.n_items) {
        if (lane == 0)
            grab = atomicAdd(a.work_next, 1ull);  // next item, in flight meanwhile
        if (!process_item<G>(kv_map, a, item, stage0, base_ptr, base_u32, bars[warp], phases, policy))
            break;
        item = __shfl_sync(0xffffffffu, grab, 0);
    }
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
    size_t off_counters, off_ml, off_o, total;
};

int make_plan(const rt_attn_params_t *p, Plan *pl)
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
        // 48 pages (768 tokens) per warp item (measured best on B200 for both
        // the ragged config-2 batch and the rollout loop); smaller when there
        // are too few items to give every warp slot of the GPU several.
        cp = 48;
        const uint64_t warp_slots = (uint64_t)rt::num_sms() * 2u * kWarps;
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
    const size_t bh = (size_t)p->num_seqs * p->num_kv_heads;
    auto up = [](size_t x) { return (x + 255u) & ~(size_t)255u; };
    pl->off_counters = 256;
    pl->off_ml = pl->off_counters + up(bh * 4u);
    pl->off_o = pl->off_ml + up(bh * pl->max_chunks * g * 2u * 4u);
    pl->total = pl->off_o + up(bh * pl->max_chunks * g * 128u * 4u);
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
                             kSmemBytes);
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
    paged_gqa_decode_kernel<G><<<grid, kWarps * 32, kSmemBytes, s>>>(map, args);
    cudaError_t e = cudaGetLastError();
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
        const uint64_t resident = (uint64_t)rt::num_sms() * 2u;
        *ctas = need < resident ? need : resident;
    }
    return RT_OK;
}

extern "C" int rt_paged_decode_attention(const rt_attn_params_t *p, const void *q,
                                         const void *kv_arena, const int32_t *page_table,
                                         const int32_t *seq_lens, float *out, void *workspace,
                                         size_t workspace_bytes, void *stream)
{
    Plan pl;
    int rc = make_plan(p, &pl);
    if (rc != RT_OK)
        return rc;
    if (!q || !kv_arena || !page_table || !seq_lens || !out || !workspace) {
        rt::set_error("attention: null pointer argument");
        return RT_EINVAL;
    }
    if (((uintptr_t)q & 3u) || ((uintptr_t)out & 3u) || ((uintptr_t)workspace & 255u) ||
        ((uintptr_t)kv_arena & 15u) || ((uintptr_t)page_table & 3u) ||
        ((uintptr_t)seq_lens & 3u)) {
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
    // Persistent grid: two CTAs per SM (the shared-memory limit), never
    // more CTAs than there are items to hand out.
    uint64_t ctas = (args.n_items + kWarps - 1) / kWarps;
    const uint64_t resident = (uint64_t)rt::num_sms() * 2u;
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

extern "C" int rt_attn_workspace_error(void *workspace, void *stream, int32_t *code)
{
    if (!workspace || !code) {
        rt::set_error("attention: null argument");
        return RT_EINVAL;
    }
    int32_t v = 0;
    cudaStream_t s = (cudaStream_t)stream;
    cudaError_t e = cudaMemcpyAsync(&v, workspace, sizeof(v), cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess)
        e = cudaStreamSynchronize(s);
    if (e == cudaSuccess)
        e = cudaMemsetAsync(workspace, 0, sizeof(v), s);
    if (e != cudaSuccess)
        return rt::cuda_fail(e, "attention: read error word");
    *code = v;
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

// Device address of g_attn_static_scratch, resolved once per device.
int static_scratch_ptr(void **out)
{
    static std::mutex mu;
    static void *ptrs[64] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess)
        return rt::cuda_fail(e, "attention_noalloc: cudaGetDevice");
    if (dev < 0 || dev >= 64) {
        rt::set_error("attention_noalloc: device index %d out of range", dev);
        return RT_EINVAL;
    }
    std::lock_guard<std::mutex> lk(mu);
    if (!ptrs[dev]) {
        void *p = nullptr;
        e = cudaGetSymbolAddress(&p, g_attn_static_scratch);
        if (e != cudaSuccess)
            return rt::cuda_fail(e, "attention_noalloc: cudaGetSymbolAddress");
        ptrs[dev] = p;
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
