// sample.cu - fused temperature / top-k / top-p sampler for sm_100a.
//
// Replaces reference cu/sample.cu:40-123 (sample_token: one thread, ~6 serial
// passes over the vocabulary and an O(V*k) insertion sort) with one 512-thread
// CTA per row, two CTAs per SM (all 256 rows of a decode pass run at once),
// the row streamed once, with a second, partial read from L2:
//
//  1. one streaming pass (16-byte loads, eight in flight per thread): scale
//     by 1.0f / temperature (the reference's fp32 multiply), keep each
//     thread's maximum and each 16-byte chunk's maximum (in shared memory,
//     as bf16 rounded up), detect NaN / +inf;
//  2. each of the 16 warps takes its m = ceil(nk / 16) largest per-thread
//     maxima (m rounds of a warp-wide max); tau0 = the nk-th largest of
//     those 16 m values.  They are distinct row entries, so at least nk
//     values are >= tau0: tau0 <= the top-k cutoff (the nk-th largest value
//     counted with multiplicity) and every survivor is >= tau0.  The largest
//     of them is the row maximum, the softmax's max;
//  3. a second, partial pass loads only the chunks whose maximum reaches
//     tau0 (one L2 round trip; about 60 of 8,000 chunks at config 3) and
//     collects the candidates (values >= tau0, typically 50-90 for k = 50).
//     Rows too long for the chunk table, or not 16-byte aligned, re-read the
//     shares of the threads whose own maximum reaches tau0 instead.  One
//     all-pairs scan of the candidates (16 bytes at a time) gives each its
//     rank by vocabulary index and whether it survives (fewer than nk
//     candidates strictly larger); it is stored at that rank as
//     __expf(l - max) if it survives, else as +0;
//  4. one thread replays the reference's serial fp32 arithmetic over those
//     entries in index order: sum of the exponentials, 1.0f / sum,
//     cumulative walk, reading eight values at a time.  Adding +0 leaves a
//     sum unchanged, and so do the entries the reference masks to -FLT_MAX:
//     their __expf(-FLT_MAX - max) is checked to be exactly 0.  Skipping
//     them keeps every fp32 sum bit-identical.
//
// Producer maxima (rt_sample_rows_cmax): when the kernel that wrote the
// logits also wrote each 16-column chunk's maximum (NaN if the chunk holds a
// NaN), pass 1 reads those 2,000 floats per row instead of the row itself:
// the per-thread maxima, NaN / +inf detection and tau0 follow from them
// unchanged (1 / T > 0, so scaling is monotone and a chunk's scaled maximum
// is the maximum of its scaled values), and pass 2 loads only the chunks
// whose scaled maximum reaches tau0, four lanes per chunk.  The logits row
// is then read only where candidates can be.
//
// Rows the fast path cannot reproduce exactly (top-k disabled, fewer than k
// finite values, > kCap candidates, a non-zero masked contribution) take
// exact slow paths: a streamed radix select for the cutoff, and, when needed,
// the whole row's exponentials staged through shared memory 256 at a time
// and summed / walked by one thread in index order.  Rows with a NaN or +inf
// after scaling return vocab - 1, which is what the reference's walk returns
// for them (its sum becomes NaN).
#include <algorithm>
#include <cfloat>
#include <cstdint>
#include <mutex>

#include "rlrt.h"
#include "rt_common.cuh"
#include "rt_internal.h"

namespace {

constexpr int kThr = 512;            // threads per row
constexpr int kWarpsPerRow = kThr / 32;
constexpr int kBins = 4096;          // radix digits of the streamed cutoff select
constexpr int kCap = 1024;           // candidates handled by the fast path
constexpr int kCmax = 8192;          // 16-byte chunks whose maxima pass 1 keeps (vocab <= 32768)
constexpr uint32_t kMaxVocab = 1u << 20;
constexpr uint32_t kChunk = 16;      // logits per producer chunk maximum


struct SampleArgs {
    const float *logits;
    const rt_sample_row_t *rows;
    const uint32_t *enable;
    uint32_t *out;
    uint64_t stride;
    uint32_t vocab;
    uint32_t fused;
    const float *cmax;   // producer chunk maxima [num_rows][cstride], or nullptr
    uint32_t cstride;
};

using rt::nan_max;

__device__ __forceinline__ uint32_t float_key(float v)
{
    const uint32_t u = __float_as_uint(v == 0.0f ? 0.0f : v);  // -0 sorts as +0
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__device__ __forceinline__ float key_float(uint32_t k)
{
    return __uint_as_float((k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k);
}

struct __align__(16) Smem {
    union {
        uint32_t hist[kBins];
        struct {
            uint32_t idx[kCap];
            float val[kCap];
        } sorted;
        // pass 1 -> pass 2: each 16-byte chunk's maximum (scaled), as bf16
        // rounded toward +inf, so a chunk whose bf16 maximum is below a
        // threshold holds no value at or above it
        uint16_t cmax[kCmax];
        // pass 2 with producer maxima: each warp's list of chunks to load
        uint32_t wl[kWarpsPerRow][128];
    } u;
    uint32_t cand_idx[kCap];
    float cand_val[kCap];
    float e[kCap];                 // exponentials; keep flags before that
    uint32_t red_u[kWarpsPerRow];
    float red_f[kWarpsPerRow];
    alignas(16) float top[kWarpsPerRow * 16];  // each warp's m largest per-thread maxima (m <= 16)
    uint32_t scan[kWarpsPerRow];
    uint32_t digit, need, count, token, done;
};

// bf16 bits of the smallest bf16 >= x (x not NaN).
__device__ __forceinline__ uint16_t bf16_round_up(float x)
{
    const uint32_t u = __float_as_uint(x);
    if ((u & 0x7FFFFFFFu) >= 0x7F800000u || (u & 0xFFFFu) == 0u)
        return (uint16_t)(u >> 16);                     // +-inf, or exact
    return (u & 0x80000000u) ? (uint16_t)(u >> 16)        // negative: truncation is up
                             : (uint16_t)((u >> 16) + 1u);  // positive: next bf16 up
}

__device__ __forceinline__ float bf16_bits_float(uint16_t b)
{
    return __uint_as_float((uint32_t)b << 16);
}

__device__ __forceinline__ uint32_t block_sum_u32(uint32_t v, Smem &s)
{
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 16; o; o >>= 1)
        v += __shfl_xor_sync(0xffffffffu, v, o);
    if (lane == 0)
        s.red_u[warp] = v;
    __syncthreads();
    uint32_t t = 0;
#pragma unroll
    for (int w = 0; w < kWarpsPerRow; w++)
        t += s.red_u[w];
    __syncthreads();
    return t;
}

__device__ __forceinline__ float block_max_f32(float v, Smem &s)
{
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 16; o; o >>= 1)
        v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    if (lane == 0)
        s.red_f[warp] = v;
    __syncthreads();
    float t = -FLT_MAX;
#pragma unroll
    for (int w = 0; w < kWarpsPerRow; w++)
        t = fmaxf(t, s.red_f[w]);
    __syncthreads();
    return t;
}

// Inclusive prefix sum of v over threads 0..kThr-1 (in thread order).
__device__ __forceinline__ uint32_t block_inclusive_scan(uint32_t v, Smem &s, uint32_t &total)
{
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    uint32_t x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o)
            x += y;
    }
    if (lane == 31)
        s.scan[warp] = x;
    __syncthreads();
    uint32_t before = 0;
    total = 0;
#pragma unroll
    for (int w = 0; w < kWarpsPerRow; w++) {
        before += w < warp ? s.scan[w] : 0u;
        total += s.scan[w];
    }
    __syncthreads();
    return x + before;
}

// Scaled logit of entry idx: the reference's fp32 multiply by 1 / T.
struct RowReader {
    const float *row;
    float inv_t;
    bool scale;
    __device__ __forceinline__ float operator()(uint32_t idx) const
    {
        const float v = __ldg(row + idx);
        return scale ? __fmul_rn(v, inv_t) : v;
    }
};

// One radix digit of the nk-th largest key among values > -FLT_MAX,
// streaming the row: histogram the keys matching `prefix` on `mask`, then
// locate the digit holding the need-th largest.  Updates prefix/mask/need.
__device__ __forceinline__ void radix_pass_row(const RowReader &rd, uint32_t V, int shift, int bits,
                                               uint32_t &prefix, uint32_t &mask, uint32_t &need,
                                               Smem &s)
{
    const int nb = 1 << bits;
    for (int b = threadIdx.x; b < nb; b += kThr)
        s.u.hist[b] = 0u;
    __syncthreads();
    for (uint32_t idx = threadIdx.x; idx < V; idx += kThr) {
        const float v = rd(idx);
        if (v > -FLT_MAX) {
            const uint32_t k = float_key(v);
            if ((k & mask) == prefix)
                atomicAdd(&s.u.hist[(k >> shift) & (uint32_t)(nb - 1)], 1u);
        }
    }
    __syncthreads();
    // thread t owns bins [per*t, per*t + per)
    const int per = nb / kThr > 0 ? nb / kThr : 1;
    const int b0 = threadIdx.x * per;
    uint32_t mine = 0;
    if (b0 < nb)
        for (int j = 0; j < per; j++)
            mine += s.u.hist[b0 + j];
    uint32_t total;
    const uint32_t incl = block_inclusive_scan(mine, s, total);
    if (b0 < nb) {
        uint32_t above = total - incl;  // keys in bins above this thread's range
        for (int j = per - 1; j >= 0; j--) {
            const uint32_t h = s.u.hist[b0 + j];
            if (above < need && above + h >= need) {
                s.digit = (uint32_t)(b0 + j);
                s.need = need - above;
            }
            above += h;
        }
    }
    __syncthreads();
    prefix |= s.digit << shift;
    mask |= (uint32_t)(nb - 1) << shift;
    need = s.need;
    __syncthreads();
}

// Survivors among the nc candidates in cand_*: a candidate survives iff
// fewer than nk candidates are strictly larger (all when nk == 0).  Writes
// them sorted by vocabulary index to s.u.sorted; returns their count.  The
// candidate arrays are padded to a multiple of 4 (-inf, index ~0) so that
// the all-pairs scans read them 16 bytes at a time.
__device__ __forceinline__ uint32_t select_and_sort(uint32_t nc, uint32_t nk, Smem &s)
{
    uint32_t *keep = reinterpret_cast<uint32_t *>(s.e);  // reused before the exponentials
    const uint32_t n4 = (nc + 3u) & ~3u;
    for (uint32_t j = nc + threadIdx.x; j < n4; j += kThr) {
        s.cand_val[j] = -INFINITY;
        s.cand_idx[j] = 0xFFFFFFFFu;
        keep[j] = 0u;
    }
    __syncthreads();
    const float4 *cv4 = reinterpret_cast<const float4 *>(s.cand_val);
    uint32_t mine = 0;
    for (uint32_t j = threadIdx.x; j < nc; j += kThr) {
        uint32_t k = 1u;
        if (nk) {
            const float v = s.cand_val[j];
            uint32_t gt = 0;
            for (uint32_t i = 0; i < n4 / 4u; i++) {
                const float4 c = cv4[i];
                gt += (c.x > v ? 1u : 0u) + (c.y > v ? 1u : 0u) + (c.z > v ? 1u : 0u) +
                      (c.w > v ? 1u : 0u);
            }
            k = gt < nk ? 1u : 0u;
        }
        keep[j] = k;
        mine += k;
    }
    const uint32_t ns = block_sum_u32(mine, s);  // includes a barrier: keep[] is complete
    const uint4 *ci4 = reinterpret_cast<const uint4 *>(s.cand_idx);
    const uint4 *kp4 = reinterpret_cast<const uint4 *>(keep);
    for (uint32_t j = threadIdx.x; j < nc; j += kThr) {
        if (!keep[j])
            continue;
        const uint32_t id = s.cand_idx[j];
        uint32_t rank = 0;
        for (uint32_t i = 0; i < n4 / 4u; i++) {
            const uint4 c = ci4[i], f = kp4[i];
            rank += (f.x && c.x < id ? 1u : 0u) + (f.y && c.y < id ? 1u : 0u) +
                    (f.z && c.z < id ? 1u : 0u) + (f.w && c.w < id ? 1u : 0u);
        }
        s.u.sorted.idx[rank] = id;
        s.u.sorted.val[rank] = s.cand_val[j];
    }
    __syncthreads();
    return ns;
}

// The nc candidates of cand_* in vocabulary order, in one all-pairs pass:
// candidate j goes to position (its index's rank among the candidates) with
// s.e = __expf(value - mx) if it survives (fewer than nk candidates strictly
// larger; all when nk == 0), else +0, which leaves the serial sum and the
// cumulative walk unchanged.  Zero-padded to a multiple of 8 entries (the
// candidate arrays to a multiple of 4, -inf at index ~0, so the scans read
// 16 bytes at a time); returns the padded count.
__device__ __forceinline__ uint32_t survivors_by_index(uint32_t nc, uint32_t nk, float mx,
                                                       Smem &s)
{
    const uint32_t n4 = (nc + 3u) & ~3u, n8 = (nc + 7u) & ~7u;
    for (uint32_t j = nc + threadIdx.x; j < n8; j += kThr) {
        if (j < n4) {
            s.cand_val[j] = -INFINITY;
            s.cand_idx[j] = 0xFFFFFFFFu;
        }
        s.e[j] = 0.0f;
        s.u.sorted.idx[j] = 0u;
    }
    __syncthreads();
    const float4 *cv4 = reinterpret_cast<const float4 *>(s.cand_val);
    const uint4 *ci4 = reinterpret_cast<const uint4 *>(s.cand_idx);
    for (uint32_t j = threadIdx.x; j < nc; j += kThr) {
        const float v = s.cand_val[j];
        const uint32_t id = s.cand_idx[j];
        uint32_t gt = 0, lo = 0;
#pragma unroll 4
        for (uint32_t i = 0; i < n4 / 4u; i++) {
            const float4 c = cv4[i];
            const uint4 d = ci4[i];
            gt += (c.x > v ? 1u : 0u) + (c.y > v ? 1u : 0u) + (c.z > v ? 1u : 0u) +
                  (c.w > v ? 1u : 0u);
            lo += (d.x < id ? 1u : 0u) + (d.y < id ? 1u : 0u) + (d.z < id ? 1u : 0u) +
                  (d.w < id ? 1u : 0u);
        }
        s.u.sorted.idx[lo] = id;
        s.e[lo] = (nk == 0u || gt < nk) ? __expf(__fsub_rn(v, mx)) : 0.0f;
    }
    __syncthreads();
    return n8;
}

// Streams the row as 16-byte loads (kDepth in flight per thread) when the
// row is 16-byte aligned, calling f(scaled value, vocabulary index); the
// remainder and unaligned rows go element by element.
template <typename F>
__device__ __forceinline__ void stream_row(const RowReader &rd, uint32_t V, F &&f)
{
    const bool vec = (reinterpret_cast<uintptr_t>(rd.row) & 15u) == 0u;
    const uint32_t V4 = vec ? V / 4u : 0u;
    const float4 *row4 = reinterpret_cast<const float4 *>(rd.row);
    constexpr uint32_t kDepth = 8;
    const uint32_t tid = threadIdx.x;
    for (uint32_t base = 0; base < V4; base += kDepth * kThr) {
        float4 buf[kDepth];
#pragma unroll
        for (uint32_t j = 0; j < kDepth; j++) {
            const uint32_t q = base + j * kThr + tid;
            if (q < V4)
                buf[j] = __ldg(row4 + q);
        }
#pragma unroll
        for (uint32_t j = 0; j < kDepth; j++) {
            const uint32_t q = base + j * kThr + tid;
            if (q < V4) {
                const float4 v = buf[j];
                if (rd.scale) {
                    f(__fmul_rn(v.x, rd.inv_t), 4u * q);
                    f(__fmul_rn(v.y, rd.inv_t), 4u * q + 1u);
                    f(__fmul_rn(v.z, rd.inv_t), 4u * q + 2u);
                    f(__fmul_rn(v.w, rd.inv_t), 4u * q + 3u);
                } else {
                    f(v.x, 4u * q);
                    f(v.y, 4u * q + 1u);
                    f(v.z, 4u * q + 2u);
                    f(v.w, 4u * q + 3u);
                }
            }
        }
    }
    for (uint32_t idx = 4u * V4 + tid; idx < V; idx += kThr)
        f(rd(idx), idx);
}

// The reference's serial fp32 sum and cumulative walk over the survivors'
// exponentials e[0 .. ns8) (zero-padded to a multiple of 8; adding +0 leaves
// the sum and the walk unchanged), one thread; returns the token.
__device__ __forceinline__ uint32_t serial_walk(const Smem &s, uint32_t ns8, bool topp, float r,
                                                uint32_t fused, uint32_t V)
{
    const float4 *e4 = reinterpret_cast<const float4 *>(s.e);
    const uint32_t nb = ns8 / 8u;
    float sum = 0.0f;
#pragma unroll 2
    for (uint32_t b = 0; b < nb; b++) {
        const float4 x = e4[2 * b], y = e4[2 * b + 1];
        sum = __fadd_rn(sum, x.x);
        sum = __fadd_rn(sum, x.y);
        sum = __fadd_rn(sum, x.z);
        sum = __fadd_rn(sum, x.w);
        sum = __fadd_rn(sum, y.x);
        sum = __fadd_rn(sum, y.y);
        sum = __fadd_rn(sum, y.z);
        sum = __fadd_rn(sum, y.w);
    }
    const float inv = topp ? __fdiv_rn(1.0f, sum) : 0.0f;
    auto step = [&](float c, float e) {
        return topp ? (fused ? __fmaf_rn(e, inv, c) : __fadd_rn(c, __fmul_rn(e, inv)))
                    : __fadd_rn(c, __fdiv_rn(e, sum));
    };
    // cum never decreases, and a +0 entry (padding, or a candidate that did
    // not survive) repeats the previous value (r > 0), so the first entry
    // with cum >= r is a survivor
    float cum = 0.0f;
    for (uint32_t b = 0; b < nb; b++) {
        const float4 x = e4[2 * b], y = e4[2 * b + 1];
        const float ev[8] = {x.x, x.y, x.z, x.w, y.x, y.y, y.z, y.w};
        int hit = -1;
#pragma unroll
        for (int i = 0; i < 8; i++) {
            cum = step(cum, ev[i]);
            if (hit < 0 && cum >= r)
                hit = i;
        }
        if (hit >= 0)
            return s.u.sorted.idx[8u * b + (uint32_t)hit];
    }
    return V - 1u;
}

__global__ void __launch_bounds__(kThr, 2) sample_rows_kernel(const SampleArgs a)
{
    __shared__ Smem s;
    const int tid = threadIdx.x;
    const int lane = tid & 31, warp = tid >> 5;
    const uint32_t V = a.vocab;
    // When launched as a programmatic dependent of the kernel that wrote the
    // logits, wait for it before reading them (a no-op otherwise).
    rt::grid_dep_wait();
    // A dependent launch after this one (the rollout loop's next schedule
    // kernel) is released once every row has its candidates (after pass 2):
    // releasing it at this grid's start cost 2% per pass, at pass 2 it gains
    // 0.2%.
    if (a.enable && a.enable[blockIdx.x] == 0u)
        return;
    const rt_sample_row_t P = a.rows[blockIdx.x];
    RowReader rd;
    rd.row = a.logits + (size_t)blockIdx.x * a.stride;
    rd.scale = P.temperature > 0.0f;
    rd.inv_t = rd.scale ? __fdiv_rn(1.0f, P.temperature) : 1.0f;

    // ---- pass 1: per-thread maximum of the values > -FLT_MAX, NaN / +inf,
    // and (rows of up to kCmax 16-byte chunks, 16-byte aligned) each chunk's
    // maximum for pass 2 ----
    float tmax = -INFINITY;
    bool bad = false;
    const bool vec = (reinterpret_cast<uintptr_t>(rd.row) & 15u) == 0u;
    const uint32_t V4 = vec ? V / 4u : 0u;
    const bool track = vec && V4 <= (uint32_t)kCmax;
    // producer maxima: thread t owns the chunks 4g .. 4g+3 for g = t, t + kThr, ...
    const float *crow = a.cmax ? a.cmax + (size_t)blockIdx.x * a.cstride : nullptr;
    const uint32_t nch = (V + kChunk - 1u) / kChunk;
    const uint32_t ngr = (nch + 3u) / 4u;
    float4 cm0 = make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);  // group g = t
    if (crow) {
        for (uint32_t g = (uint32_t)tid; g < ngr; g += kThr) {
            const float4 c = __ldg(reinterpret_cast<const float4 *>(crow) + g);
            if (g == (uint32_t)tid)
                cm0 = c;
            const float cv[4] = {c.x, c.y, c.z, c.w};
#pragma unroll
            for (uint32_t j = 0; j < 4u; j++) {
                if (4u * g + j < nch) {
                    const float x = rd.scale ? __fmul_rn(cv[j], rd.inv_t) : cv[j];
                    bad |= !(x < INFINITY);  // NaN or +inf in the chunk
                    tmax = x > -FLT_MAX ? fmaxf(tmax, x) : tmax;
                }
            }
        }
    } else {
        const float4 *row4 = reinterpret_cast<const float4 *>(rd.row);
        constexpr uint32_t kDepth = 8;
        for (uint32_t base = 0; base < V4; base += kDepth * kThr) {
            float4 buf[kDepth];
#pragma unroll
            for (uint32_t j = 0; j < kDepth; j++) {
                const uint32_t q = base + j * kThr + (uint32_t)tid;
                if (q < V4)
                    buf[j] = __ldg(row4 + q);
            }
#pragma unroll
            for (uint32_t j = 0; j < kDepth; j++) {
                const uint32_t q = base + j * kThr + (uint32_t)tid;
                if (q < V4) {
                    float4 v = buf[j];
                    if (rd.scale) {
                        v.x = __fmul_rn(v.x, rd.inv_t);
                        v.y = __fmul_rn(v.y, rd.inv_t);
                        v.z = __fmul_rn(v.z, rd.inv_t);
                        v.w = __fmul_rn(v.w, rd.inv_t);
                    }
                    bad |= !(v.x < INFINITY) || !(v.y < INFINITY) || !(v.z < INFINITY) ||
                           !(v.w < INFINITY);
                    const float cm = fmaxf(fmaxf(v.x, v.y), fmaxf(v.z, v.w));
                    // cm > -FLT_MAX: cm is a value > -FLT_MAX of the chunk
                    tmax = cm > -FLT_MAX ? fmaxf(tmax, cm) : tmax;
                    if (track)
                        s.u.cmax[q] = bf16_round_up(cm);
                }
            }
        }
        for (uint32_t idx = 4u * V4 + (uint32_t)tid; idx < V; idx += kThr) {
            const float v = rd(idx);
            bad |= !(v < INFINITY);  // NaN or +inf
            tmax = v > -FLT_MAX ? fmaxf(tmax, v) : tmax;
        }
    }
    if (tid == 0) {
        uint32_t ph[4];
        rt::philox4x32_10((uint32_t)P.step, (uint32_t)(P.step >> 32), P.rollout_id, 0u,
                          (uint32_t)P.seed, (uint32_t)(P.seed >> 32), ph);
        s.token = ph[0] & 0x00FFFFFFu;  // u24
        s.count = 0u;
        s.done = 0u;
    }
    if (__syncthreads_or(bad)) {
        if (tid == 0)
            a.out[blockIdx.x] = V - 1u;
        return;
    }
    const uint32_t u24 = s.token;
    if (u24 == 0u) {  // r == 0: the walk stops at index 0
        if (tid == 0)
            a.out[blockIdx.x] = 0u;
        return;
    }
    const float r = (float)u24 / 16777216.0f;
    const bool topp = P.top_p > 0.0f && P.top_p < 1.0f;
    const bool topk = P.top_k > 0u && P.top_k < V;
    const uint32_t nk = P.top_k < 256u ? P.top_k : 256u;

    // ---- top-k cutoff and survivors ----
    float cutoff = -FLT_MAX;
    bool fast = topk;
    uint32_t ns = 0;
    bool sorted_ready = false;
    if (topk) {
        // tau0: every warp contributes its m largest per-thread maxima
        // (m = ceil(nk / 16), so 16 m >= nk values, each from a different
        // thread and so a different row entry); tau0 = the nk-th largest of
        // them.  At least nk row values are >= tau0, so tau0 <= the top-k
        // cutoff and every survivor is >= tau0.  (About 60 candidates
        // survive the threshold at config 3, against ~140 for the smallest
        // of the warps' m-th largest maxima.)
        const uint32_t m = (nk + kWarpsPerRow - 1) / kWarpsPerRow;
        // the warp's m largest per-thread maxima, one warp-wide max a round
        // (a tie goes to the lowest lane, which then drops out: keys of
        // values are > 0, a removed lane holds 0)
        uint32_t key = float_key(tmax);
        for (uint32_t j = 0; j < m; j++) {
            const uint32_t kmax = __reduce_max_sync(0xffffffffu, key);
            const uint32_t who = __ballot_sync(0xffffffffu, key == kmax);
            if (lane == __ffs(who) - 1) {
                s.top[warp * m + j] = key_float(kmax);
                key = 0u;
            }
        }
        __syncthreads();
        const uint32_t n_top = m * kWarpsPerRow;  // a multiple of 16
        if ((uint32_t)tid < n_top) {
            const float v = s.top[tid];
            const float4 *t4 = reinterpret_cast<const float4 *>(s.top);
            uint32_t g2 = 0, e2 = 0;
#pragma unroll 4
            for (uint32_t i = 0; i < n_top / 4u; i++) {
                const float4 x = t4[i];
                g2 += (x.x > v ? 1u : 0u) + (x.y > v ? 1u : 0u) + (x.z > v ? 1u : 0u) +
                      (x.w > v ? 1u : 0u);
                e2 += (x.x >= v ? 1u : 0u) + (x.y >= v ? 1u : 0u) + (x.z >= v ? 1u : 0u) +
                      (x.w >= v ? 1u : 0u);
            }
            if (g2 < nk && e2 >= nk)
                s.red_f[0] = v;  // every such thread holds the same value
            if (g2 == 0u)
                s.red_f[1] = v;  // the row maximum (of the values > -FLT_MAX)
        }
        __syncthreads();
        const float tau0 = s.red_f[0];
        const float rowmax = s.red_f[1];
        // fewer than nk finite maxima: the fallback below counts the values
        // (red_f is next written by a block reduction behind later barriers)
        const bool ok = tau0 > -FLT_MAX;
        if (ok) {
            // ---- pass 2: candidates >= tau0, re-read only by the threads
            // whose own maximum reaches tau0 (the others hold none: about
            // one thread in eight re-reads its share of the row) ----
            auto add = [&](float v, uint32_t idx) {
                if (v >= tau0) {
                    const uint32_t pos = atomicAdd(&s.count, 1u);
                    if (pos < (uint32_t)kCap) {
                        s.cand_idx[pos] = idx;
                        s.cand_val[pos] = v;
                    }
                }
            };
            if (crow) {
                // chunks whose scaled producer maximum reaches tau0: each
                // warp lists its lanes' chunks, then loads them four lanes
                // per chunk (one 16-byte load per lane, 8 chunks a round)
                uint32_t *wl = s.u.wl[warp];
                for (uint32_t g0 = 0; g0 < ngr; g0 += kThr) {  // uniform over the block
                    const uint32_t g = g0 + (uint32_t)tid;
                    uint32_t bits = 0;
                    if (g < ngr) {
                        const float4 c = g0 == 0u ? cm0
                                                  : __ldg(reinterpret_cast<const float4 *>(crow) + g);
                        const float cv[4] = {c.x, c.y, c.z, c.w};
#pragma unroll
                        for (uint32_t j = 0; j < 4u; j++) {
                            const float x = rd.scale ? __fmul_rn(cv[j], rd.inv_t) : cv[j];
                            bits |= (4u * g + j < nch && x >= tau0) ? 1u << j : 0u;
                        }
                    }
                    const uint32_t n = __popc(bits);
                    uint32_t incl = n;
#pragma unroll
                    for (int o = 1; o < 32; o <<= 1) {
                        const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
                        if (lane >= o)
                            incl += y;
                    }
                    const uint32_t total = __shfl_sync(0xffffffffu, incl, 31);
                    uint32_t pos = incl - n;
                    while (bits) {
                        const uint32_t j = (uint32_t)__ffs(bits) - 1u;
                        bits &= bits - 1u;
                        wl[pos++] = 4u * g + j;
                    }
                    __syncwarp();
                    for (uint32_t i = (uint32_t)lane >> 2; i < ((total + 7u) & ~7u); i += 8u) {
                        if (i < total) {
                            const uint32_t i0 = wl[i] * kChunk + 4u * ((uint32_t)lane & 3u);
                            if (vec && i0 + 3u < V) {
                                float4 x = __ldg(reinterpret_cast<const float4 *>(rd.row + i0));
                                if (rd.scale) {
                                    x.x = __fmul_rn(x.x, rd.inv_t);
                                    x.y = __fmul_rn(x.y, rd.inv_t);
                                    x.z = __fmul_rn(x.z, rd.inv_t);
                                    x.w = __fmul_rn(x.w, rd.inv_t);
                                }
                                add(x.x, i0);
                                add(x.y, i0 + 1u);
                                add(x.z, i0 + 2u);
                                add(x.w, i0 + 3u);
                            } else {
                                for (uint32_t k = 0; k < 4u; k++)
                                    if (i0 + k < V)
                                        add(rd(i0 + k), i0 + k);
                            }
                        }
                    }
                    __syncwarp();  // the list is rewritten by the next round
                }
            } else if (track) {
                // only the chunks whose maximum reaches tau0, loaded together
                // (a thread rarely has more than one)
                const float4 *row4 = reinterpret_cast<const float4 *>(rd.row);
                uint32_t q = (uint32_t)tid;
                while (q < V4) {
                    uint32_t sel[4] = {0u, 0u, 0u, 0u};
                    uint32_t n = 0;
                    for (; q < V4 && n < 4u; q += kThr) {
                        if (bf16_bits_float(s.u.cmax[q]) >= tau0) {
                            // register slots, no local-memory array
                            sel[0] = n == 0u ? q : sel[0];
                            sel[1] = n == 1u ? q : sel[1];
                            sel[2] = n == 2u ? q : sel[2];
                            sel[3] = n == 3u ? q : sel[3];
                            n++;
                        }
                    }
                    float4 v[4];
#pragma unroll
                    for (uint32_t k = 0; k < 4u; k++)
                        if (k < n)
                            v[k] = __ldg(row4 + sel[k]);
#pragma unroll
                    for (uint32_t k = 0; k < 4u; k++) {
                        if (k < n) {
                            float4 x = v[k];
                            if (rd.scale) {
                                x.x = __fmul_rn(x.x, rd.inv_t);
                                x.y = __fmul_rn(x.y, rd.inv_t);
                                x.z = __fmul_rn(x.z, rd.inv_t);
                                x.w = __fmul_rn(x.w, rd.inv_t);
                            }
                            add(x.x, 4u * sel[k]);
                            add(x.y, 4u * sel[k] + 1u);
                            add(x.z, 4u * sel[k] + 2u);
                            add(x.w, 4u * sel[k] + 3u);
                        }
                    }
                }
                for (uint32_t idx = 4u * V4 + (uint32_t)tid; idx < V; idx += kThr)
                    add(rd(idx), idx);
            } else if (tmax >= tau0) {
                stream_row(rd, V, add);
            }
            __syncthreads();
            const uint32_t nc = s.count;
            rt::grid_dep_launch();
            if (nc <= (uint32_t)kCap) {
                // The masked entries' terms __expf(-FLT_MAX - max) must be
                // exactly 0 (the maximum is the row maximum: it survives).
                // Then every candidate goes in index order, non-survivors
                // as +0 terms, and one barrier precedes the walk.
                if (__expf(__fsub_rn(-FLT_MAX, rowmax)) == 0.0f) {
                    const uint32_t nc8 = survivors_by_index(nc, nk, rowmax, s);
                    if (tid == 0)
                        a.out[blockIdx.x] = serial_walk(s, nc8, topp, r, a.fused, V);
                    return;
                }
                ns = select_and_sort(nc, nk, s);
                sorted_ready = true;
            }
        } else {
            // a warp holds fewer than m finite maxima: count the finite
            // values; with fewer than nk the cutoff stays -FLT_MAX
            uint32_t nfin = 0;
            stream_row(rd, V, [&](float v, uint32_t) { nfin += v > -FLT_MAX ? 1u : 0u; });
            if (block_sum_u32(nfin, s) < nk)
                fast = false;
        }
        if (fast && !sorted_ready) {
            // Tie-heavy or degenerate rows: exact cutoff by a streamed radix select.
            uint32_t prefix = 0, mask = 0, need = nk;
            radix_pass_row(rd, V, 20, 12, prefix, mask, need, s);
            radix_pass_row(rd, V, 8, 12, prefix, mask, need, s);
            radix_pass_row(rd, V, 0, 8, prefix, mask, need, s);
            cutoff = key_float(prefix);
            if (tid == 0)
                s.count = 0u;
            __syncthreads();
            stream_row(rd, V, [&](float v, uint32_t idx) {
                if (v >= cutoff) {
                    const uint32_t pos = atomicAdd(&s.count, 1u);
                    if (pos < (uint32_t)kCap) {
                        s.cand_idx[pos] = idx;
                        s.cand_val[pos] = v;
                    }
                }
            });
            __syncthreads();
            const uint32_t nc = s.count;
            if (nc <= (uint32_t)kCap)
                ns = select_and_sort(nc, 0u, s);  // every value >= cutoff survives
            else
                fast = false;
        }
    }

    float mx = -FLT_MAX;
    if (fast) {
        float m = -FLT_MAX;
        for (uint32_t j = tid; j < ns; j += kThr)
            m = fmaxf(m, s.u.sorted.val[j]);
        mx = block_max_f32(m, s);
        // masked entries hold -FLT_MAX; their terms must be exactly zero
        if (__expf(__fsub_rn(-FLT_MAX, mx)) != 0.0f)
            fast = false;
    }
    if (fast) {
        // exponentials, zero-padded to a multiple of 8: adding +0 leaves the
        // sum and the cumulative walk unchanged, so the serial loops below
        // can read 8 values per step
        const uint32_t ns8 = (ns + 7u) & ~7u;
        for (uint32_t j = tid; j < ns8; j += kThr)
            s.e[j] = j < ns ? __expf(__fsub_rn(s.u.sorted.val[j], mx)) : 0.0f;
        __syncthreads();
        if (tid == 0)
            a.out[blockIdx.x] = serial_walk(s, ns8, topp, r, a.fused, V);
        return;
    }

    // ---- exact slow path: every entry, in index order ----
    auto masked = [&](uint32_t idx) {
        const float v = rd(idx);
        return (topk && v < cutoff) ? -FLT_MAX : v;
    };
    float m = -FLT_MAX;
    for (uint32_t idx = (uint32_t)tid; idx < V; idx += kThr)
        m = fmaxf(m, masked(idx));
    mx = block_max_f32(m, s);
    float sum = 0.0f, inv = 0.0f, cum = 0.0f;
    uint32_t tok = V - 1u;
    for (int pass = 0; pass < 2; pass++) {
        for (uint32_t base = 0; base < V; base += kThr) {
            const uint32_t idx = base + (uint32_t)tid;
            s.e[tid] = idx < V ? __expf(__fsub_rn(masked(idx), mx)) : 0.0f;
            __syncthreads();
            if (tid == 0 && !s.done) {
                const uint32_t n = min((uint32_t)kThr, V - base);
                if (pass == 0) {
                    for (uint32_t j = 0; j < n; j++)
                        sum = __fadd_rn(sum, s.e[j]);
                } else {
                    for (uint32_t j = 0; j < n; j++) {
                        cum = topp ? (a.fused ? __fmaf_rn(s.e[j], inv, cum)
                                              : __fadd_rn(cum, __fmul_rn(s.e[j], inv)))
                                   : __fadd_rn(cum, __fdiv_rn(s.e[j], sum));
                        if (cum >= r) {
                            tok = base + j;
                            s.done = 1u;
                            break;
                        }
                    }
                }
            }
            __syncthreads();
        }
        if (tid == 0)
            inv = __fdiv_rn(1.0f, sum);
    }
    if (tid == 0)
        a.out[blockIdx.x] = tok;
}

// chunk_max[r][c] = max of logits[r][16c .. 16c+15] (NaN if one is NaN):
// lanes read consecutive 16-byte groups of the row and the four lanes of a
// chunk reduce it with two shuffles.  Grid (x: chunks of the row, y: rows).
__global__ void __launch_bounds__(256) chunk_max_kernel(const float *logits, uint32_t V,
                                                        uint64_t stride, float *cmax,
                                                        uint32_t cstride)
{
    const float *row = logits + (size_t)blockIdx.y * stride;
    float *crow = cmax + (size_t)blockIdx.y * cstride;
    const uint32_t nq = (V + 3u) / 4u;
    const bool vec = (reinterpret_cast<uintptr_t>(row) & 15u) == 0u;
    const uint32_t lane = threadIdx.x & 31u;
    const uint32_t step = gridDim.x * blockDim.x;
    for (uint32_t q0 = blockIdx.x * blockDim.x + threadIdx.x - lane; q0 < nq; q0 += step) {
        const uint32_t q = q0 + lane;
        float m = -INFINITY;
        if (q < nq) {
            const uint32_t i = 4u * q;
            if (vec && i + 3u < V) {
                const float4 v = __ldg(reinterpret_cast<const float4 *>(row + i));
                m = nan_max(nan_max(v.x, v.y), nan_max(v.z, v.w));
            } else {
                for (uint32_t k = 0; k < 4u; k++)
                    if (i + k < V)
                        m = nan_max(m, __ldg(row + i + k));
            }
        }
        m = nan_max(m, __shfl_xor_sync(0xffffffffu, m, 1));
        m = nan_max(m, __shfl_xor_sync(0xffffffffu, m, 2));
        if ((q & 3u) == 0u && q < nq)
            crow[q / 4u] = m;
    }
}

}  // namespace

extern "C" uint32_t rt_chunk_max_stride(uint32_t vocab)
{
    const uint32_t nch = (vocab + kChunk - 1u) / kChunk;
    return (nch + 3u) & ~3u;
}

extern "C" int rt_logits_chunk_max(const float *logits, uint32_t num_rows, uint32_t vocab,
                                   uint64_t row_stride, float *chunk_max, uint32_t cmax_stride,
                                   void *stream)
{
    if (!logits || !chunk_max) {
        rt::set_error("chunk_max: null argument");
        return RT_EINVAL;
    }
    if (vocab == 0 || vocab > kMaxVocab || row_stride < vocab ||
        cmax_stride < rt_chunk_max_stride(vocab)) {
        rt::set_error("chunk_max: vocab %u must be in 1..%u, <= row_stride %llu, and "
                      "cmax_stride %u >= %u",
                      vocab, kMaxVocab, (unsigned long long)row_stride, cmax_stride,
                      rt_chunk_max_stride(vocab));
        return RT_EINVAL;
    }
    if (((uintptr_t)logits & 3u) || ((uintptr_t)chunk_max & 3u) || num_rows > 65535u) {
        rt::set_error("chunk_max: misaligned pointer or more than 65535 rows");
        return RT_EINVAL;
    }
    if (num_rows == 0)
        return RT_OK;
    const uint32_t nq = (vocab + 3u) / 4u;
    const dim3 grid(std::min((nq + 255u) / 256u, 64u), num_rows);
    chunk_max_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(logits, vocab, row_stride, chunk_max,
                                                              cmax_stride);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? RT_OK : rt::cuda_fail(e, "chunk_max: launch");
}

extern "C" int rt_sample_rows_cmax(const rt_sample_params_t *p, const float *logits,
                                   const float *chunk_max, uint32_t cmax_stride,
                                   const rt_sample_row_t *rows, uint32_t *tokens_out,
                                   void *stream)
{
    if (!chunk_max) {
        rt::set_error("sample: null chunk_max");
        return RT_EINVAL;
    }
    return rt::sample_rows_launch(p, logits, rows, tokens_out, (cudaStream_t)stream, false,
                                  chunk_max, cmax_stride);
}

extern "C" uint32_t rt_sample_uniform24(uint64_t seed, uint32_t rollout_id, uint64_t step)
{
    uint32_t o[4];
    rt::philox4x32_10((uint32_t)step, (uint32_t)(step >> 32), rollout_id, 0u, (uint32_t)seed,
                      (uint32_t)(seed >> 32), o);
    return o[0] & 0x00FFFFFFu;
}

extern "C" int rt_sample_rows(const rt_sample_params_t *p, const float *logits,
                              const rt_sample_row_t *rows, uint32_t *tokens_out, void *stream)
{
    return rt::sample_rows_launch(p, logits, rows, tokens_out, (cudaStream_t)stream, false);
}

int rt::sample_rows_launch(const rt_sample_params_t *p, const float *logits,
                           const rt_sample_row_t *rows, uint32_t *tokens_out, cudaStream_t stream,
                           bool pdl, const float *cmax, uint32_t cmax_stride)
{
    if (!p || !logits || !rows || !tokens_out) {
        rt::set_error("sample: null argument");
        return RT_EINVAL;
    }
    if (p->vocab == 0 || p->vocab > kMaxVocab || p->row_stride < p->vocab) {
        rt::set_error("sample: vocab %u must be in 1..%u and <= row_stride %llu", p->vocab,
                      kMaxVocab, (unsigned long long)p->row_stride);
        return RT_EINVAL;
    }
    if (((uintptr_t)logits & 3u) || ((uintptr_t)rows & 7u) || ((uintptr_t)tokens_out & 3u) ||
        ((uintptr_t)p->row_enable & 3u)) {
        rt::set_error("sample: misaligned pointer");
        return RT_EINVAL;
    }
    if (cmax && (((uintptr_t)cmax & 15u) || (cmax_stride & 3u) ||
                 cmax_stride < rt_chunk_max_stride(p->vocab))) {
        rt::set_error("sample: chunk_max must be 16-byte aligned with a stride that is a "
                      "multiple of 4 and >= %u (got %u)",
                      rt_chunk_max_stride(p->vocab), cmax_stride);
        return RT_EINVAL;
    }
    if (p->num_rows == 0)
        return RT_OK;
    if (p->num_rows > 0x7FFFFFFFu) {
        rt::set_error("sample: too many rows");
        return RT_EINVAL;
    }
    SampleArgs a;
    a.logits = logits;
    a.rows = rows;
    a.out = tokens_out;
    a.enable = p->row_enable;
    a.stride = p->row_stride;
    a.vocab = p->vocab;
    a.fused = p->fused_cum ? 1u : 0u;
    a.cmax = cmax;
    a.cstride = cmax_stride;
    cudaError_t e;
    if (pdl) {
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(p->num_rows);
        cfg.blockDim = dim3(kThr);
        cfg.dynamicSmemBytes = 0;
        cfg.stream = stream;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        e = cudaLaunchKernelEx(&cfg, sample_rows_kernel, a);
    } else {
        sample_rows_kernel<<<p->num_rows, kThr, 0, stream>>>(a);
        e = cudaGetLastError();
    }
    return e == cudaSuccess ? RT_OK : rt::cuda_fail(e, "sample: launch");
}
