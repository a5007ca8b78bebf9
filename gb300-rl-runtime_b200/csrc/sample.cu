// sample.cu - fused temperature / top-k / top-p sampler for sm_100a.
//
// Replaces reference cu/sample.cu:40-123 (sample_token: one thread, ~6 serial
// passes over the vocabulary and an O(V*k) insertion sort) with one CTA of
// 1024 threads per row that reads the row's logits from HBM exactly once
// and keeps them in registers (32 per thread, vocab <= 32768):
//
//  1. scale by 1.0f / temperature (same fp32 multiply as the reference);
//  2. exact top-k cutoff = the k-th largest value (with multiplicity) by a
//     three-pass radix select (12 + 12 + 8 bits) on order-preserving keys,
//     shared-memory histograms, block-wide suffix scans;
//  3. survivors (value >= cutoff, ties included) are compacted and sorted
//     by vocabulary index (rank sort, typically k of them);
//  4. one thread replays the reference's serial fp32 arithmetic over the
//     survivors only: sum of __expf(l - max) in index order, 1.0f / sum,
//     cumulative walk.  Entries the reference masks to -FLT_MAX contribute
//     __expf(-FLT_MAX - max) which is checked to be exactly 0, so skipping
//     them leaves every fp32 sum bit-identical.
//
// Rows the fast path cannot reproduce exactly (top-k disabled, fewer than k
// finite values, > 2048 survivors, a non-zero masked contribution) take an
// exact slow path: the whole row's exponentials are staged through shared
// memory 1024 at a time and one thread sums / walks them in index order.
// Rows with a NaN or +inf after scaling return vocab - 1, which is what the
// reference's walk returns for them (its sum becomes NaN).
#include <cfloat>
#include <cstdint>

#include "rlrt.h"
#include "rt_common.cuh"

namespace {

constexpr int kThreads = 1024;
constexpr int kItems = 32;          // vocab <= kThreads * kItems
constexpr int kBins = 4096;
constexpr int kCap = 2048;          // survivors handled by the fast path

struct SampleArgs {
    const float *logits;
    const rt_sample_row_t *rows;
    const uint32_t *enable;
    uint32_t *out;
    uint64_t stride;
    uint32_t vocab;
    uint32_t fused;
};

__device__ __forceinline__ uint32_t float_key(float v)
{
    const uint32_t u = __float_as_uint(v == 0.0f ? 0.0f : v);  // -0 sorts as +0
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__device__ __forceinline__ float key_float(uint32_t k)
{
    return __uint_as_float((k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k);
}

struct Smem {
    union {
        uint32_t hist[kBins];
        struct {
            uint32_t idx[kCap];
            float val[kCap];
        } sorted;
    } u;
    uint32_t surv_idx[kCap];
    float surv_val[kCap];
    float e[kCap];
    uint32_t red_u[32];
    float red_f[32];
    uint32_t scan[32];
    uint32_t digit, need, count, token, done;
};

__device__ __forceinline__ uint32_t block_sum_u32(uint32_t v, Smem &s)
{
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 16; o; o >>= 1)
        v += __shfl_xor_sync(0xffffffffu, v, o);
    if (lane == 0)
        s.red_u[warp] = v;
    __syncthreads();
    uint32_t t = lane < (int)(blockDim.x >> 5) ? s.red_u[lane] : 0u;
#pragma unroll
    for (int o = 16; o; o >>= 1)
        t += __shfl_xor_sync(0xffffffffu, t, o);
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
    float t = lane < (int)(blockDim.x >> 5) ? s.red_f[lane] : -FLT_MAX;
#pragma unroll
    for (int o = 16; o; o >>= 1)
        t = fmaxf(t, __shfl_xor_sync(0xffffffffu, t, o));
    __syncthreads();
    return t;
}

// Inclusive prefix sum of v over threads 0..blockDim-1 (in thread order).
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
    if (warp == 0) {
        uint32_t w = s.scan[lane];
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const uint32_t y = __shfl_up_sync(0xffffffffu, w, o);
            if (lane >= o)
                w += y;
        }
        s.scan[lane] = w;
    }
    __syncthreads();
    total = s.scan[31];
    const uint32_t r = x + (warp ? s.scan[warp - 1] : 0u);
    __syncthreads();
    return r;
}

// One radix digit: histogram the keys of candidates that match `prefix` on
// `mask`, then find the digit d holding the need-th largest key.  Updates
// prefix/mask/need for the next digit.
template <int N>
__device__ __forceinline__ void radix_pass(const float (&x)[N], int shift, int bits,
                                           uint32_t &prefix, uint32_t &mask, uint32_t &need,
                                           Smem &s)
{
    const int nb = 1 << bits;
    for (int b = threadIdx.x; b < nb; b += kThreads)
        s.u.hist[b] = 0u;
    __syncthreads();
#pragma unroll
    for (int i = 0; i < N; i++) {
        if (x[i] > -FLT_MAX) {  // entries past the vocabulary hold -inf
            const uint32_t k = float_key(x[i]);
            if ((k & mask) == prefix)
                atomicAdd(&s.u.hist[(k >> shift) & (uint32_t)(nb - 1)], 1u);
        }
    }
    __syncthreads();
    // thread t owns bins [per*t, per*t + per)
    const int per = nb / kThreads > 0 ? nb / kThreads : 1;
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

__global__ void __launch_bounds__(kThreads, 1) sample_rows_kernel(const SampleArgs a)
{
    __shared__ Smem s;
    const int tid = threadIdx.x;
    const uint32_t V = a.vocab;
    if (a.enable && a.enable[blockIdx.x] == 0u)
        return;
    const rt_sample_row_t P = a.rows[blockIdx.x];
    const float *lr = a.logits + (size_t)blockIdx.x * a.stride;

    // ---- 1. load once, temperature ----
    const bool scale = P.temperature > 0.0f;
    const float inv_t = scale ? __fdiv_rn(1.0f, P.temperature) : 1.0f;
    // x[i] = entry tid + i * kThreads; entries past the vocabulary hold -inf,
    // which is never a top-k candidate, never a survivor and never the max.
    float x[kItems];
    bool bad = false;
#pragma unroll
    for (int i = 0; i < kItems; i++) {
        const uint32_t idx = (uint32_t)tid + (uint32_t)i * kThreads;
        float v = -INFINITY;
        if (idx < V) {
            v = __ldg(lr + idx);
            if (scale)
                v = __fmul_rn(v, inv_t);
            bad |= isnan(v) || v == INFINITY;
        }
        x[i] = v;
    }

    if (tid == 0) {
        uint32_t ph[4];
        rt::philox4x32_10((uint32_t)P.step, (uint32_t)(P.step >> 32), P.rollout_id, 0u,
                          (uint32_t)P.seed, (uint32_t)(P.seed >> 32), ph);
        s.token = ph[0] & 0x00FFFFFFu;  // u24 (reused below)
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

    // ---- 2. top-k cutoff and survivors ----
    // A value survives iff it is >= the nk-th largest value (counted with
    // multiplicity) among values > -FLT_MAX, i.e. iff fewer than nk values
    // are strictly greater than it.
    float cutoff = -FLT_MAX;
    bool fast = topk;
    uint32_t ns = 0;
    bool sorted_ready = false;
    if (topk) {
        uint32_t ncand = 0;
#pragma unroll
        for (int i = 0; i < kItems; i++)
            ncand += x[i] > -FLT_MAX ? 1u : 0u;
        ncand = block_sum_u32(ncand, s);
        if (ncand < nk)
            fast = false;  // cutoff stays -FLT_MAX; almost everything survives
    }
    if (fast) {
        // Quick path: tau0 = the nk-th largest of the 1024 per-thread maxima.
        // Those maxima are nk distinct entries >= tau0, so tau0 <= cutoff and
        // every survivor is among the few entries >= tau0.
        float tm[1] = {-INFINITY};
#pragma unroll
        for (int i = 0; i < kItems; i++)
            if (x[i] > -FLT_MAX)
                tm[0] = fmaxf(tm[0], x[i]);
        const uint32_t nvalid = (uint32_t)__syncthreads_count(tm[0] > -FLT_MAX);
        if (nvalid >= nk) {
            uint32_t prefix = 0, mask = 0, need = nk;
            radix_pass(tm, 20, 12, prefix, mask, need, s);
            radix_pass(tm, 8, 12, prefix, mask, need, s);
            radix_pass(tm, 0, 8, prefix, mask, need, s);
            const float tau0 = key_float(prefix);
            if (tid == 0)
                s.count = 0u;
            __syncthreads();
#pragma unroll
            for (int i = 0; i < kItems; i++) {
                if (x[i] >= tau0 && x[i] > -FLT_MAX) {
                    const uint32_t pos = atomicAdd(&s.count, 1u);
                    if (pos < (uint32_t)kCap) {
                        s.surv_idx[pos] = (uint32_t)tid + (uint32_t)i * kThreads;
                        s.surv_val[pos] = x[i];
                    }
                }
            }
            __syncthreads();
            const uint32_t nc = s.count;
            if (nc <= (uint32_t)kCap) {
                uint32_t *keep = reinterpret_cast<uint32_t *>(s.e);  // reused before the walk
                uint32_t mine = 0;
                for (uint32_t j = tid; j < nc; j += kThreads) {
                    const float v = s.surv_val[j];
                    uint32_t gt = 0;
                    for (uint32_t i2 = 0; i2 < nc; i2++)
                        gt += s.surv_val[i2] > v ? 1u : 0u;
                    keep[j] = gt < nk ? 1u : 0u;
                    mine += keep[j];
                }
                ns = block_sum_u32(mine, s);  // includes a barrier: keep[] is complete
                for (uint32_t j = tid; j < nc; j += kThreads) {
                    if (!keep[j])
                        continue;
                    const uint32_t id = s.surv_idx[j];
                    uint32_t rank = 0;
                    for (uint32_t i2 = 0; i2 < nc; i2++)
                        rank += (keep[i2] && s.surv_idx[i2] < id) ? 1u : 0u;
                    s.u.sorted.idx[rank] = id;
                    s.u.sorted.val[rank] = s.surv_val[j];
                }
                sorted_ready = true;
            }
        }
        if (!sorted_ready) {
            // Tie-heavy or degenerate rows: exact cutoff by a full-row radix select.
            uint32_t prefix = 0, mask = 0, need = nk;
            radix_pass(x, 20, 12, prefix, mask, need, s);
            radix_pass(x, 8, 12, prefix, mask, need, s);
            radix_pass(x, 0, 8, prefix, mask, need, s);
            cutoff = key_float(prefix);
        }
    }

    // ---- 3. survivors, sorted by index ----
    float mx = -FLT_MAX;
    if (fast && !sorted_ready) {
        if (tid == 0)
            s.count = 0u;
        __syncthreads();
#pragma unroll
        for (int i = 0; i < kItems; i++) {
            if (x[i] >= cutoff) {
                const uint32_t pos = atomicAdd(&s.count, 1u);
                if (pos < (uint32_t)kCap) {
                    s.surv_idx[pos] = (uint32_t)tid + (uint32_t)i * kThreads;
                    s.surv_val[pos] = x[i];
                }
            }
        }
        __syncthreads();
        ns = s.count;
        if (ns > (uint32_t)kCap)
            fast = false;
        if (fast) {
            for (uint32_t j = tid; j < ns; j += kThreads) {
                const uint32_t id = s.surv_idx[j];
                uint32_t rank = 0;
                for (uint32_t q = 0; q < ns; q++)
                    rank += s.surv_idx[q] < id ? 1u : 0u;
                s.u.sorted.idx[rank] = id;
                s.u.sorted.val[rank] = s.surv_val[j];
            }
        }
    }
    if (fast) {
        __syncthreads();  // sorted survivors complete
        float m = -FLT_MAX;
        for (uint32_t j = tid; j < ns; j += kThreads)
            m = fmaxf(m, s.u.sorted.val[j]);
        mx = block_max_f32(m, s);
        // masked entries hold -FLT_MAX; their terms must be exactly zero
        if (__expf(__fsub_rn(-FLT_MAX, mx)) != 0.0f)
            fast = false;
    }
    if (fast) {
        for (uint32_t j = tid; j < ns; j += kThreads)
            s.e[j] = __expf(__fsub_rn(s.u.sorted.val[j], mx));
        __syncthreads();
        if (tid == 0) {
            float sum = 0.0f;
            for (uint32_t j = 0; j < ns; j++)
                sum = __fadd_rn(sum, s.e[j]);
            uint32_t tok = V - 1u;
            float cum = 0.0f;
            if (topp) {
                const float inv = __fdiv_rn(1.0f, sum);
                for (uint32_t j = 0; j < ns; j++) {
                    cum = a.fused ? __fmaf_rn(s.e[j], inv, cum)
                                  : __fadd_rn(cum, __fmul_rn(s.e[j], inv));
                    if (cum >= r) {
                        tok = s.u.sorted.idx[j];
                        break;
                    }
                }
            } else {
                for (uint32_t j = 0; j < ns; j++) {
                    cum = __fadd_rn(cum, __fdiv_rn(s.e[j], sum));
                    if (cum >= r) {
                        tok = s.u.sorted.idx[j];
                        break;
                    }
                }
            }
            a.out[blockIdx.x] = tok;
        }
        return;
    }

    // ---- 4. exact slow path: every entry, in index order ----
    float m = -FLT_MAX;
#pragma unroll
    for (int i = 0; i < kItems; i++) {
        if ((uint32_t)tid + (uint32_t)i * kThreads < V) {
            if (topk && x[i] < cutoff)
                x[i] = -FLT_MAX;
            m = fmaxf(m, x[i]);
        }
    }
    mx = block_max_f32(m, s);
    float sum = 0.0f, inv = 0.0f, cum = 0.0f;
    uint32_t tok = V - 1u;
    for (int pass = 0; pass < 2; pass++) {
#pragma unroll
        for (int i = 0; i < kItems; i++) {
            if ((uint32_t)i * kThreads >= V)
                break;
            s.e[tid] = (uint32_t)tid + (uint32_t)i * kThreads < V ? __expf(__fsub_rn(x[i], mx)) : 0.0f;
            __syncthreads();
            if (tid == 0 && !s.done) {
                const uint32_t n = min((uint32_t)kThreads, V - (uint32_t)i * kThreads);
                if (pass == 0) {
                    for (uint32_t j = 0; j < n; j++)
                        sum = __fadd_rn(sum, s.e[j]);
                } else {
                    for (uint32_t j = 0; j < n; j++) {
                        cum = topp ? (a.fused ? __fmaf_rn(s.e[j], inv, cum)
                                              : __fadd_rn(cum, __fmul_rn(s.e[j], inv)))
                                   : __fadd_rn(cum, __fdiv_rn(s.e[j], sum));
                        if (cum >= r) {
                            tok = (uint32_t)i * kThreads + j;
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

}  // namespace

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
    if (!p || !logits || !rows || !tokens_out) {
        rt::set_error("sample: null argument");
        return RT_EINVAL;
    }
    if (p->vocab == 0 || p->vocab > (uint32_t)(kThreads * kItems) || p->row_stride < p->vocab) {
        rt::set_error("sample: vocab %u must be in 1..%d and <= row_stride %llu", p->vocab,
                      kThreads * kItems, (unsigned long long)p->row_stride);
        return RT_EINVAL;
    }
    if (((uintptr_t)logits & 3u) || ((uintptr_t)rows & 7u) || ((uintptr_t)tokens_out & 3u) ||
        ((uintptr_t)p->row_enable & 3u)) {
        rt::set_error("sample: misaligned pointer");
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
    sample_rows_kernel<<<p->num_rows, kThreads, 0, (cudaStream_t)stream>>>(a);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? RT_OK : rt::cuda_fail(e, "sample: launch");
}
