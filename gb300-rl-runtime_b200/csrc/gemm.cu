// gemm.cu - bf16 GEMM on the 5th-generation tensor cores (tcgen05, sm_100a)
// for the decode step's projections: C[m][n] = sum_k A[m][k] * B[n][k],
// A = activations (one row per rollout slot), B = a weight matrix stored
// [out][in] (K contiguous), C fp32.
//
// Reference: none.  The reference synthesises its decode query with one
// <<<1, 128>>> launch per slot and step (cu/model_state.cu:6-52,
// cu/query_producer.cu:5-26) and has no LM head; this is the batched
// projection those per-slot launches stand in for.
//
// Kernel: one persistent CTA per SM walking (tile, K-split) units of
// 256 x 224 outputs: the decode batch (256 slots) is one M tile, so each
// CTA fetches its weight slab exactly once and 32,000 / 224 gives 143
// units, one wave on 148 SMs.  Three warp roles:
//   warp 0   one thread issues TMA loads of the A (256 x 64) and B
//            (224 x 64) K-slices into a 3-stage shared-memory ring
//            (60 KiB per stage, 128-byte swizzle, no multicast);
//   warp 1   allocates 512 TMEM columns (two fp32 accumulators of 128
//            lanes x 224 columns, one per 128-row half of the tile) and
//            one thread issues tcgen05.mma (M 128, N 224, K 16: two halves
//            x four per K-slice, sharing the B slice), committing each
//            stage back to the producer and each finished unit to the
//            epilogue;
//   warps 2-9  read the accumulators out of TMEM (tcgen05.ld, one row per
//            thread, four warps per half) and store C.
// With K-splits every split stores its partial tile into a workspace
// [split][M][N] in parallel, and a second kernel sums the partials in
// split order into C: results do not depend on scheduling, and no split
// waits for another.
// Every mbarrier wait is bounded; an expired wait sets the error word and
// the CTA winds down (waiting, bounded, for its own MMAs) and frees its TMEM.
#include <algorithm>
#include <cuda_bf16.h>
#include <stdint.h>
#include <string.h>

#include "rlrt.h"
#include "rt_common.cuh"
#include "rt_internal.h"

namespace {

#ifndef RT_GEMM_BK
#define RT_GEMM_BK 64
#endif
// K-slice per stage: 64 bf16 (128-byte rows, 128-byte swizzle, 3 stages of
// 60 KiB) or 32 (64-byte rows, 64-byte swizzle, 6 stages of 30 KiB).
constexpr uint32_t kBM = 256, kBN = 224, kBK = RT_GEMM_BK, kStages = kBK == 64u ? 3u : 6u;
constexpr uint32_t kRowBytes = kBK * 2u;                   // one operand row of a stage
constexpr uint32_t kAtomBytes = 8u * kRowBytes;            // 8-row swizzle atom
constexpr uint32_t kSwizzleMode = kBK == 64u ? 2u : 4u;    // descriptor layout: 128B / 64B
static_assert(kBK == 64u || kBK == 32u, "K-slice of 32 or 64");
constexpr uint32_t kHalf = 128;                      // rows per UMMA (M 128)
constexpr uint32_t kABytes = kBM * kBK * 2;         // 32 KiB
constexpr uint32_t kBBytes = kBN * kBK * 2;         // 28 KiB
constexpr uint32_t kStageBytes = kABytes + kBBytes;  // multiple of 1024 (swizzle atoms)
constexpr uint32_t kAccCols = 256;                   // TMEM columns per accumulator (half)
constexpr uint32_t kTmemCols = 2 * kAccCols;
constexpr uint32_t kThreads = 320;
constexpr uint64_t kWaitNs = 2000000000ull;
constexpr uint32_t kOutBytes = kBM * 32u * 4u;      // one 32-column fp32 slab of a tile
constexpr uint32_t kSmemBytes = kStages * kStageBytes + kOutBytes + 1024 /* alignment */ +
                                256 /* barriers */;


static_assert(kABytes % 1024 == 0 && kBBytes % 1024 == 0, "stage buffers stay 1024-byte aligned");
static_assert(kBN % 16 == 0 && kBN <= 256 && kBN <= kAccCols, "UMMA N for M = 128");

struct GemmArgs {
    float *C;
    float *ws;  // K-split partials [splits][m_tiles * 256][N] (splits > 1)
    uint32_t M, N, K, ldc;
    uint32_t tma_out;  // 1: the output goes out through map_c (TMA tensor stores)
    uint32_t m_tiles, n_tiles, splits, kb_per_split, kb_total;
    uint32_t units;
    uint32_t accumulate;  // 1: add into C (K-splits always add)
    uint32_t vec_ok;      // the output rows allow 16-byte stores
    int32_t *error;
    float *cmax;          // each row's 16-column maxima (written with the final C), or nullptr
    uint32_t cstride;
};

// The 16-column maxima of the 32 columns n .. n+31 of row m that a thread
// holds (n a multiple of 16): NaN if a column is NaN, columns past N left out.
__device__ __forceinline__ void store_chunk_max(const GemmArgs &g, uint32_t m, uint32_t n,
                                                const uint32_t (&r)[32])
{
    if (m >= g.M)
        return;
    if (n + 32u <= g.N) {
        // a full slab: two 16-wide trees, no column checks
        float t[16];
#pragma unroll
        for (uint32_t half = 0; half < 2u; half++) {
#pragma unroll
            for (uint32_t j = 0; j < 8u; j++)
                t[j] = rt::nan_max(__uint_as_float(r[16u * half + 2u * j]),
                                   __uint_as_float(r[16u * half + 2u * j + 1u]));
#pragma unroll
            for (uint32_t w = 4u; w >= 1u; w >>= 1)
#pragma unroll
                for (uint32_t j = 0; j < w; j++)
                    t[j] = rt::nan_max(t[2u * j], t[2u * j + 1u]);
            g.cmax[(size_t)m * g.cstride + n / 16u + half] = t[0];
        }
        return;
    }
#pragma unroll
    for (uint32_t half = 0; half < 2u; half++) {
        const uint32_t n0 = n + 16u * half;
        if (n0 >= g.N)
            break;
        float mx = -INFINITY;
#pragma unroll
        for (uint32_t j = 0; j < 16u; j++)
            if (n0 + j < g.N)
                mx = rt::nan_max(mx, __uint_as_float(r[16u * half + j]));
        g.cmax[(size_t)m * g.cstride + n0 / 16u] = mx;
    }
}

struct Shared {
    uint64_t full[kStages], empty[kStages];
    uint64_t acc_full, acc_empty;
    uint32_t tmem_base;
    uint32_t abort;
    uint32_t ep_ok[8];  // epilogue warps' wait outcomes for the current unit
};

__device__ __forceinline__ void unit_coords(const GemmArgs &g, uint32_t u, uint32_t &m0,
                                            uint32_t &n0, uint32_t &kb0, uint32_t &kb1)
{
    // tiles sharing a B slab (same n) are adjacent, so concurrently running
    // CTAs read each weight slab from HBM once
    const uint32_t split = u % g.splits;
    const uint32_t t = u / g.splits;
    m0 = (t % g.m_tiles) * kBM;
    n0 = (t / g.m_tiles) * kBN;
    kb0 = split * g.kb_per_split;
    kb1 = min(kb0 + g.kb_per_split, g.kb_total);
}

// Barrier of the 256 epilogue threads (warps 2-9) only.
__device__ __forceinline__ void epilogue_sync()
{
    asm volatile("bar.sync 1, 256;" ::: "memory");
}

// K-major operand descriptor of a stage: swizzled rows of kRowBytes,
// 8-row atoms kAtomBytes apart (16 bf16 = 32 bytes further along a row per
// MMA K step).
__device__ __forceinline__ uint64_t umma_desc(uint32_t smem_addr)
{
    uint64_t d = 0;
    d |= (uint64_t)((smem_addr >> 4) & 0x3FFFu);
    d |= (uint64_t)(16u >> 4) << 16;
    d |= (uint64_t)((kAtomBytes >> 4) & 0x3FFFu) << 32;
    d |= (uint64_t)1u << 46;  // version
    d |= (uint64_t)kSwizzleMode << 61;
    return d;
}

__device__ __forceinline__ bool wait_or_abort(Shared *sh, uint32_t bar, uint32_t parity,
                                              const GemmArgs &g)
{
    if (rt::mbar_try_wait(bar, parity))
        return true;
    const uint64_t t0 = rt::globaltimer_ns();
    while (!rt::mbar_try_wait(bar, parity)) {
        if (*(volatile uint32_t *)&sh->abort)
            return false;
        if (rt::globaltimer_ns() - t0 > kWaitNs) {
            atomicCAS(g.error, 0, 1);
            *(volatile uint32_t *)&sh->abort = 1u;
            return false;
        }
    }
    return true;
}

// TMA tensor store / reduce-add of a shared-memory box (bulk-group completion).
__device__ __forceinline__ void tma_store_2d(const CUtensorMap *map, uint32_t src, int32_t x,
                                             int32_t y, bool add)
{
    if (add)
        asm volatile(
            "cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.tile.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
                map),
            "r"(x), "r"(y), "r"(src)
            : "memory");
    else
        asm volatile(
            "cp.async.bulk.tensor.2d.global.shared::cta.tile.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
                map),
            "r"(x), "r"(y), "r"(src)
            : "memory");
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

__global__ void __launch_bounds__(kThreads, 1)
    gemm_bf16_tn_kernel(const __grid_constant__ CUtensorMap map_a,
                        const __grid_constant__ CUtensorMap map_b,
                        const __grid_constant__ CUtensorMap map_c, const GemmArgs g)
{
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023u) & ~uintptr_t(1023u));
    uint8_t *out_buf = smem + kStages * kStageBytes;  // 1024-aligned, 128-byte swizzled rows
    Shared *sh = reinterpret_cast<Shared *>(out_buf + kOutBytes);
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    const uint32_t smem_base = rt::smem_u32(smem);

    if (threadIdx.x == 0) {
        for (uint32_t s = 0; s < kStages; s++) {
            rt::mbar_init(rt::smem_u32(&sh->full[s]), 1u);
            rt::mbar_init(rt::smem_u32(&sh->empty[s]), 1u);
        }
        rt::mbar_init(rt::smem_u32(&sh->acc_full), 1u);
        rt::mbar_init(rt::smem_u32(&sh->acc_empty), 256u);
        sh->abort = 0u;
        rt::mbar_fence_init();
        rt::prefetch_tensormap(&map_a);
        rt::prefetch_tensormap(&map_b);
    }
    if (warp == 1) {
        rt::tmem_alloc(rt::smem_u32(&sh->tmem_base), kTmemCols);
        rt::tmem_relinquish();
    }
    rt::tc_fence_before_sync();
    __syncthreads();
    rt::tc_fence_after_sync();
    const uint32_t tmem = sh->tmem_base;

    if (warp == 0) {
        // ---------------------------------------------------- TMA producer
        if (lane == 0) {
            uint32_t stage = 0, phase = 0;
            for (uint32_t u = blockIdx.x; u < g.units; u += gridDim.x) {
                uint32_t m0, n0, kb0, kb1;
                unit_coords(g, u, m0, n0, kb0, kb1);
                bool ok = true;
                for (uint32_t kb = kb0; kb < kb1; kb++) {
                    if (!(ok = wait_or_abort(sh, rt::smem_u32(&sh->empty[stage]), phase ^ 1u, g)))
                        break;
                    const uint32_t full = rt::smem_u32(&sh->full[stage]);
                    const uint32_t sa = smem_base + stage * kStageBytes;
                    rt::mbar_arrive_expect_tx(full, kStageBytes);
                    rt::tma_load_2d(sa, &map_a, (int32_t)(kb * kBK), (int32_t)m0, full,
                                    rt::l2_policy_evict_normal());
                    rt::tma_load_2d(sa + kABytes, &map_b, (int32_t)(kb * kBK), (int32_t)n0, full,
                                    rt::l2_policy_evict_first());
                    if (++stage == kStages) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                if (!ok)
                    break;
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------ MMA issuer
        if (lane == 0) {
            const uint32_t idesc = rt::umma_idesc_bf16(kHalf, kBN, 0u);
            uint32_t stage = 0, phase = 0, acc_phase = 0;
            for (uint32_t u = blockIdx.x; u < g.units; u += gridDim.x) {
                uint32_t m0, n0, kb0, kb1;
                unit_coords(g, u, m0, n0, kb0, kb1);
                const uint32_t halves = m0 + kHalf < g.M ? 2u : 1u;  // rows past M: no MMA
                if (!wait_or_abort(sh, rt::smem_u32(&sh->acc_empty), acc_phase ^ 1u, g))
                    break;
                rt::tc_fence_after_sync();
                bool ok = true;
                for (uint32_t kb = kb0; kb < kb1; kb++) {
                    if (!(ok = wait_or_abort(sh, rt::smem_u32(&sh->full[stage]), phase, g)))
                        break;
                    rt::tc_fence_after_sync();
                    const uint32_t sa = smem_base + stage * kStageBytes;
#pragma unroll
                    for (uint32_t kk = 0; kk < kBK / 16u; kk++) {
                        // K-major SW128: 16 bf16 = 32 bytes further along each row
                        const uint64_t db = umma_desc(sa + kABytes + kk * 32u);
                        for (uint32_t h = 0; h < halves; h++) {
                            const uint64_t da = umma_desc(sa + h * (kHalf * kRowBytes) + kk * 32u);
                            rt::umma_bf16_ss(tmem + h * kAccCols, da, db, idesc,
                                             (kb > kb0 || kk > 0u) ? 1u : 0u);
                        }
                    }
                    rt::umma_commit(rt::smem_u32(&sh->empty[stage]));
                    if (++stage == kStages) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                if (!ok)
                    break;
                rt::umma_commit(rt::smem_u32(&sh->acc_full));
                acc_phase ^= 1u;
            }
        }
    } else {
        // ------------------------------------------------------- epilogue
        const uint32_t quarter = warp & 3u;  // TMEM lanes 32*quarter .. +31
        const uint32_t half = (warp - 2u) >> 2;
        const uint32_t row = half * kHalf + quarter * 32u + lane;
        uint32_t acc_phase = 0;
        for (uint32_t u = blockIdx.x; u < g.units; u += gridDim.x) {
            uint32_t m0, n0, kb0, kb1;
            unit_coords(g, u, m0, n0, kb0, kb1);
            const uint32_t split = u % g.splits;
            // Exits are decided uniformly by all 256 epilogue threads (the
            // TMEM loads are warp-collective and the named barriers need
            // every epilogue warp): one lane per warp waits, the outcomes
            // meet in shared memory, everyone reads them after a barrier.
            bool ok = true;
            if (lane == 0u)
                ok = wait_or_abort(sh, rt::smem_u32(&sh->acc_full), acc_phase, g);
            if (lane == 0u)
                sh->ep_ok[warp - 2u] = ok ? 1u : 0u;
            epilogue_sync();
            bool go = true;
#pragma unroll
            for (uint32_t w = 0; w < 8u; w++)
                go &= sh->ep_ok[w] != 0u;
            if (!go)
                break;
            rt::tc_fence_after_sync();
            const uint32_t m = m0 + row;
            // a K-split stores its partial tile into its workspace slice
            const uint32_t m_pad = g.m_tiles * kBM;
            float *crow = g.splits > 1u ? g.ws + ((uint64_t)split * m_pad + m) * g.N
                                        : g.C + (uint64_t)m * g.ldc;
            const bool add = g.accumulate && g.splits == 1u;
            if (g.tma_out) {
                // 32-column slabs: each thread writes its row into the
                // swizzled buffer, one thread stores the 256 x 32 box
                const uint32_t y = g.splits > 1u ? split * m_pad + m0 : m0;
                uint8_t *my_row = out_buf + row * 128u;
#pragma unroll 1
                for (uint32_t c = 0; c < kBN; c += 32u) {
                    uint32_t r[32];
                    rt::tmem_ld32(tmem + half * kAccCols + ((quarter * 32u) << 16) + c, r);
                    rt::tmem_ld_wait();
#pragma unroll
                    for (uint32_t j = 0; j < 8u; j++)
                        *reinterpret_cast<uint4 *>(my_row + ((j ^ (row & 7u)) << 4)) =
                            make_uint4(r[4 * j], r[4 * j + 1], r[4 * j + 2], r[4 * j + 3]);
                    rt::fence_proxy_async_smem();
                    epilogue_sync();
                    if (warp == 2u && lane == 0u) {
                        if (n0 + c < g.N)
                            tma_store_2d(&map_c, rt::smem_u32(out_buf), (int32_t)(n0 + c),
                                         (int32_t)y, add);
                        // the buffer is reused by the next slab
                        asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
                    }
                    // the chunk maxima from registers while the store drains
                    if (g.cmax)
                        store_chunk_max(g, m, n0 + c, r);
                    epilogue_sync();
                }
            } else
#pragma unroll 1
            for (uint32_t c = 0; c < kBN; c += 32u) {
                uint32_t r[32];
                rt::tmem_ld32(tmem + half * kAccCols + ((quarter * 32u) << 16) + c, r);
                rt::tmem_ld_wait();
                if (g.cmax)
                    store_chunk_max(g, m, n0 + c, r);
                if (m < g.M) {
                    const uint32_t n = n0 + c;
                    if (n + 32u <= g.N && g.vec_ok) {
                        float4 *dst = reinterpret_cast<float4 *>(crow + n);
#pragma unroll
                        for (uint32_t j = 0; j < 8; j++) {
                            float4 v = make_float4(__uint_as_float(r[4 * j]), __uint_as_float(r[4 * j + 1]),
                                                   __uint_as_float(r[4 * j + 2]),
                                                   __uint_as_float(r[4 * j + 3]));
                            if (add) {
                                const float4 c = __ldcg(dst + j);
                                v = make_float4(c.x + v.x, c.y + v.y, c.z + v.z, c.w + v.w);
                            }
                            dst[j] = v;
                        }
                    } else {
#pragma unroll
                        for (uint32_t j = 0; j < 32; j++) {
                            if (n + j < g.N) {
                                const float v = __uint_as_float(r[j]);
                                crow[n + j] = add ? __ldcg(crow + n + j) + v : v;
                            }
                        }
                    }
                }
            }
            rt::tc_fence_before_sync();
            rt::mbar_arrive(rt::smem_u32(&sh->acc_empty));
            acc_phase ^= 1u;
            // every warp has read ep_ok before it is rewritten for the next unit
            epilogue_sync();
        }
    }

    // wind down: every MMA this CTA issued has completed before TMEM is
    // freed, and every tensor store has completed before the CTA exits
    if (warp == 2u && lane == 0u)
        asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
    rt::tc_fence_before_sync();
    __syncthreads();
    if (warp == 1) {
        rt::tc_fence_after_sync();
        rt::tmem_dealloc(tmem, kTmemCols);
    }
}

// C = (C if accumulating) + sum over splits of the partials, in split order.
__global__ void __launch_bounds__(256) split_reduce_kernel(float *C, uint32_t ldc,
                                                           const float *ws, uint32_t M,
                                                           uint32_t N, uint32_t splits,
                                                           uint32_t accumulate, uint32_t m_pad)
{
    const uint64_t MN = (uint64_t)M * N;
    const uint64_t slice = (uint64_t)m_pad * N;  // one split's partials (rows padded to tiles)
    if ((N & 3u) == 0u && (ldc & 3u) == 0u && ((uintptr_t)C & 15u) == 0u) {
        const uint64_t n4 = MN / 4u;
        for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n4;
             i += (uint64_t)gridDim.x * blockDim.x) {
            const uint64_t e = i * 4u, m = e / N, n = e % N;
            float4 v = __ldcg(reinterpret_cast<const float4 *>(ws) + i);
            for (uint32_t sp = 1; sp < splits; sp++) {
                const float4 w = __ldcg(reinterpret_cast<const float4 *>(ws + sp * slice) + i);
                v = make_float4(v.x + w.x, v.y + w.y, v.z + w.z, v.w + w.w);
            }
            float4 *dst = reinterpret_cast<float4 *>(C + m * ldc + n);
            if (accumulate) {
                const float4 c = *dst;
                v = make_float4(c.x + v.x, c.y + v.y, c.z + v.z, c.w + v.w);
            }
            *dst = v;
        }
        return;
    }
    for (uint64_t e = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; e < MN;
         e += (uint64_t)gridDim.x * blockDim.x) {
        float v = ws[e];
        for (uint32_t sp = 1; sp < splits; sp++)
            v += ws[sp * slice + e];
        float *dst = C + (e / N) * ldc + e % N;
        *dst = accumulate ? *dst + v : v;
    }
}

// Shared-memory opt-in of the kernel on the current device (once per
// device) and the device's SM count.
int gemm_setup(int *sms_out)
{
    static int sms_of[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) {
        rt::set_error("gemm_bf16: device index %d out of range", dev);
        return RT_EINVAL;
    }
    int &sms = sms_of[dev];
    if (!sms) {
        cudaError_t err = cudaFuncSetAttribute(
            gemm_bf16_tn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes);
        if (err == cudaSuccess)
            err = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (err != cudaSuccess) {
            sms = 0;
            return rt::cuda_fail(err, "gemm_bf16: setup");
        }
    }
    *sms_out = sms;
    return RT_OK;
}

}  // namespace

namespace rt {
int gemm_prepare()
{
    int sms = 0;
    return gemm_setup(&sms);
}
}  // namespace rt

// K-splits the call will use (after clamping to the K-slices).
static uint32_t effective_splits(const rt_gemm_params_t *p)
{
    const uint32_t kb_total = p->K / kBK;
    const uint32_t splits = p->split_k ? std::min(p->split_k, kb_total) : 1u;
    const uint32_t per = (kb_total + splits - 1) / splits;
    return (kb_total + per - 1) / per;
}

extern "C" size_t rt_gemm_workspace_bytes(const rt_gemm_params_t *p)
{
    if (!p || p->K == 0 || p->K % kBK)
        return 0;
    const uint32_t splits = effective_splits(p);
    const size_t m_pad = (size_t)((p->M + kBM - 1) / kBM) * kBM;
    return splits > 1u ? (size_t)splits * m_pad * p->N * sizeof(float) : 0u;
}

static int gemm_launch(const rt_gemm_params_t *p, const void *A, const void *B, float *C,
                       void *workspace, size_t workspace_bytes, int32_t *error, float *cmax,
                       uint32_t cmax_stride, void *stream)
{
    if (!p || !A || !B || !C || !error) {
        rt::set_error("gemm_bf16: null argument");
        return RT_EINVAL;
    }
    if (p->M == 0 || p->N == 0 || p->K == 0)
        return RT_OK;
    if (p->K % kBK || p->lda < p->K || p->ldb < p->K || p->ldc < p->N || (p->lda % 8u) ||
        (p->ldb % 8u) || ((uintptr_t)A % 16u) || ((uintptr_t)B % 16u) || ((uintptr_t)C % 4u)) {
        rt::set_error("gemm_bf16: K must be a multiple of 64, lda/ldb multiples of 8 elements "
                      "(>= K), ldc >= N, A and B 16-byte aligned (M %u N %u K %u)",
                      p->M, p->N, p->K);
        return RT_EINVAL;
    }
    CUtensorMap ma, mb;
    int rc = rt::encode_bf16_kmajor_map(&ma, A, p->K, p->M, (uint64_t)p->lda * 2u, kBM, kBK);
    if (rc == RT_OK)
        rc = rt::encode_bf16_kmajor_map(&mb, B, p->K, p->N, (uint64_t)p->ldb * 2u, kBN, kBK);
    if (rc != RT_OK)
        return rc;
    GemmArgs g;
    memset(&g, 0, sizeof(g));
    g.C = C;
    g.M = p->M;
    g.N = p->N;
    g.K = p->K;
    g.ldc = p->ldc;
    g.m_tiles = (p->M + kBM - 1) / kBM;
    g.n_tiles = (p->N + kBN - 1) / kBN;
    g.kb_total = p->K / kBK;
    const uint32_t splits = p->split_k ? min(p->split_k, g.kb_total) : 1u;
    g.kb_per_split = (g.kb_total + splits - 1) / splits;
    g.splits = (g.kb_total + g.kb_per_split - 1) / g.kb_per_split;  // no empty split
    if (g.splits > 1u) {
        const size_t need = (size_t)g.splits * g.m_tiles * kBM * p->N * sizeof(float);
        if (!workspace || workspace_bytes < need || ((uintptr_t)workspace % 16u)) {
            rt::set_error("gemm_bf16: %u K-splits need a 16-byte aligned workspace of %zu bytes",
                          g.splits, need);
            return RT_ENOMEM;
        }
        g.ws = static_cast<float *>(workspace);
    }
    g.units = g.m_tiles * g.n_tiles * g.splits;
    g.accumulate = p->flags & RT_GEMM_ACCUMULATE;
    g.error = error;
    // chunk maxima: from the epilogue when it writes the final C, else by a
    // pass over C afterwards
    const bool cmax_fused = cmax && g.splits == 1u && !g.accumulate;
    g.cmax = cmax_fused ? cmax : nullptr;
    g.cstride = cmax_stride;
    g.vec_ok = g.splits > 1u ? (p->N % 4u) == 0u
                             : ((uintptr_t)C % 16u) == 0u && (p->ldc % 4u) == 0u;
    // TMA stores need 16-byte aligned rows; otherwise plain stores
    CUtensorMap mc;
    memset(&mc, 0, sizeof(mc));
    g.tma_out = 0u;
    if (g.vec_ok) {
        const int rc3 = g.splits > 1u
                            ? rt::encode_f32_store_map(&mc, g.ws, p->N, (uint64_t)g.splits * g.m_tiles * kBM,
                                                       (uint64_t)p->N * 4u, kBM)
                            : rt::encode_f32_store_map(&mc, C, p->N, p->M, (uint64_t)p->ldc * 4u, kBM);
        if (rc3 != RT_OK)
            return rc3;
        g.tma_out = 1u;
    }
    cudaStream_t s = (cudaStream_t)stream;
    cudaError_t err;
    int sms = 0;
    int rc2 = gemm_setup(&sms);
    if (rc2 != RT_OK)
        return rc2;
    const uint32_t grid = min(g.units, (uint32_t)sms);
    gemm_bf16_tn_kernel<<<grid, kThreads, kSmemBytes, s>>>(ma, mb, mc, g);
    err = cudaGetLastError();
    if (err != cudaSuccess)
        return rt::cuda_fail(err, "gemm_bf16: launch");
    if (g.splits > 1u) {
        const uint64_t work = (uint64_t)p->M * p->N / 4u;
        const uint32_t blocks = (uint32_t)std::min<uint64_t>((work + 255u) / 256u, 4u * (uint64_t)sms);
        split_reduce_kernel<<<std::max(blocks, 1u), 256, 0, s>>>(C, p->ldc, g.ws, p->M, p->N,
                                                                 g.splits, g.accumulate,
                                                                 g.m_tiles * kBM);
        err = cudaGetLastError();
        if (err != cudaSuccess)
            return rt::cuda_fail(err, "gemm_bf16: split reduction launch");
    }
    if (cmax && !cmax_fused)
        return rt_logits_chunk_max(C, p->M, p->N, p->ldc, cmax, cmax_stride, stream);
    return RT_OK;
}

extern "C" int rt_gemm_bf16(const rt_gemm_params_t *p, const void *A, const void *B, float *C,
                            void *workspace, size_t workspace_bytes, int32_t *error, void *stream)
{
    return gemm_launch(p, A, B, C, workspace, workspace_bytes, error, nullptr, 0u, stream);
}

extern "C" int rt_gemm_bf16_chunk_max(const rt_gemm_params_t *p, const void *A, const void *B,
                                      float *C, void *workspace, size_t workspace_bytes,
                                      int32_t *error, float *chunk_max, uint32_t cmax_stride,
                                      void *stream)
{
    if (!chunk_max || ((uintptr_t)chunk_max & 3u) || !p ||
        cmax_stride < rt_chunk_max_stride(p->N)) {
        rt::set_error("gemm_bf16_chunk_max: chunk_max must be 4-byte aligned with a stride "
                      ">= rt_chunk_max_stride(N)");
        return RT_EINVAL;
    }
    return gemm_launch(p, A, B, C, workspace, workspace_bytes, error, chunk_max, cmax_stride,
                       stream);
}
