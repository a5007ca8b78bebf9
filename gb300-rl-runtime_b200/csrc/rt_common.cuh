// rt_common.cuh - sm_100a device building blocks shared by the kernels:
// shared-memory mbarriers, TMA tensor loads (no multicast), ldmatrix, bf16
// mma.sync, exp2, bounded waits, the Philox4x32-10 counter generator, and
// host-side helpers (error reporting, tensor-map encoding, device queries).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

namespace rt {

// ------------------------------------------------------------------ device
__device__ __forceinline__ uint32_t smem_u32(const void *p)
{
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer_ns()
{
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_fence_init()
{
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes)
{
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar)
{
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity)
{
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0u;
}

// Non-blocking probe of a phase (test_wait never suspends the thread, unlike
// try_wait): for a producer polling several barriers.
__device__ __forceinline__ bool mbar_test_wait(uint32_t bar, uint32_t parity)
{
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0u;
}

// Wait for the phase of `bar` with the given parity; gives up after
// `limit_ns` of wall time and returns false (the caller reports an error
// instead of hanging the GPU).
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity, uint64_t limit_ns)
{
    if (mbar_try_wait(bar, parity))
        return true;
    const uint64_t t0 = globaltimer_ns();
    while (!mbar_try_wait(bar, parity)) {
        if (globaltimer_ns() - t0 > limit_ns)
            return false;
    }
    return true;
}

// Order this thread's generic-proxy shared-memory accesses before later
// async-proxy (TMA) accesses of the same memory.
__device__ __forceinline__ void fence_proxy_async_smem()
{
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// 2-D tiled TMA load into this CTA's shared memory, completion signalled on
// an mbarrier as transaction bytes.  Plain (non-multicast) form only.
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap *map, int32_t x,
                                            int32_t y, uint32_t bar, uint64_t policy)
{
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(dst),
        "l"(map), "r"(x), "r"(y), "r"(bar), "l"(policy)
        : "memory");
}

__device__ __forceinline__ uint64_t l2_policy_evict_first()
{
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}

__device__ __forceinline__ uint64_t l2_policy_evict_last()
{
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
    return p;
}

__device__ __forceinline__ uint64_t l2_policy_evict_normal()
{
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_normal.b64 %0, 1.0;" : "=l"(p));
    return p;
}

__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap *map)
{
    asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2,
                                        uint32_t &r3)
{
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr)
                 : "memory");
}

__device__ __forceinline__ void ldsm_x4_trans(uint32_t addr, uint32_t &r0, uint32_t &r1,
                                              uint32_t &r2, uint32_t &r3)
{
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr)
                 : "memory");
}

// D += A(16x16, row) * B(16x8, col), bf16 inputs, fp32 accumulate.
__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                               uint32_t b1)
{
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
        "{%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Transpose of an 8x8 b16 matrix held as a warp fragment (thread t owns
// row t/4, columns 2(t%4), 2(t%4)+1) into the same fragment layout.
__device__ __forceinline__ uint32_t movmatrix_trans(uint32_t x)
{
    uint32_t y;
    asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
    return y;
}

// Programmatic dependent launch: a kernel launched with the programmatic
// stream-serialization attribute may start before its predecessor in the
// stream has finished; grid_dep_wait() blocks until that predecessor has
// completed and its memory is visible (a no-op for an ordinary launch), and
// grid_dep_launch() lets the next such kernel start early.
__device__ __forceinline__ void grid_dep_wait()
{
    asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void grid_dep_launch()
{
    asm volatile("griddepcontrol.launch_dependents;");
}

// ---------------------------------------------------------------- tcgen05
// Tensor memory (TMEM) and the 5th-generation tensor-core MMA.  Formats
// follow the PTX ISA for sm_100a: shared-memory matrix descriptors (start
// >> 4 at [0,14), leading byte offset >> 4 at [16,30), stride byte offset
// >> 4 at [32,46), version 1 at [46,48), layout at [61,64)) and the
// kind::f16 instruction descriptor.

// Allocate `ncols` TMEM columns (power of two >= 32) for this CTA; one full
// warp executes it.  The TMEM address is written to shared memory at dst.
__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols)
{
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish()
{
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols)
{
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tc_fence_before_sync()
{
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after_sync()
{
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// SWIZZLE_128B shared-memory matrix descriptor (version 1, base offset 0).
// K-major operand: rows of 128 bytes, 8-row groups 1024 bytes apart.
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t smem_addr, uint32_t lbo_bytes,
                                                     uint32_t sbo_bytes)
{
    uint64_t d = 0;
    d |= (uint64_t)((smem_addr >> 4) & 0x3FFFu);
    d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16;
    d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32;
    d |= (uint64_t)1u << 46;  // version
    d |= (uint64_t)2u << 61;  // SWIZZLE_128B
    return d;
}

// kind::f16 instruction descriptor: bf16 A and B, fp32 accumulator, A
// K-major, B K-major (b_mn_major = 0) or MN-major (1), M x N.
__host__ __device__ constexpr uint32_t umma_idesc_bf16(uint32_t M, uint32_t N, uint32_t b_mn_major)
{
    return (1u << 4)              // D format: f32
           | (1u << 7)            // A format: bf16
           | (1u << 10)           // B format: bf16
           | (b_mn_major << 16)   // B major
           | ((N >> 3) << 17)     // N / 8
           | ((M >> 4) << 24);    // M / 16
}

// D[tmem] (+)= A[smem desc] * B[smem desc]; issued by one thread.
__device__ __forceinline__ void umma_bf16_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                             uint32_t idesc, uint32_t accumulate)
{
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrive on a shared-memory mbarrier once this thread's earlier tcgen05.mma
// operations have completed.
__device__ __forceinline__ void umma_commit(uint32_t bar)
{
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                 : "memory");
}

// 32 consecutive TMEM columns of this warp's 32 lanes (lane i of the warp
// reads TMEM lane taddr.lane + i); complete after tmem_ld_wait().
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32])
{
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
          "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
          "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
          "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait()
{
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// 2^x with the SFU (ex2.approx, flush-to-zero); 2^-inf = +0.
__device__ __forceinline__ float fast_exp2(float x)
{
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// How paged decode attention splits a sequence into items: its own pages
// are those past the group-covered prefix (skip), in chunks of chunk_pages;
// chunk 0 holds the remainder and every other chunk is full.  A fully
// covered sequence still has chunk 0, which folds the group's partials into
// the output.  An invalid length gives no pages and an invalid skip counts
// as 0 (the attention kernel flags both).  The rollout loop's schedule
// kernel evaluates the same function to publish each pass's largest chunk
// count.
struct AttnSeqShape {
    int n_pages, skip, n_chunks;
    uint32_t n_g;
    bool bad_len, bad_skip;
};
__host__ __device__ __forceinline__ AttnSeqShape attn_seq_shape(int L, uint32_t skip_raw,
                                                                uint32_t max_seq_len,
                                                                uint32_t max_pages,
                                                                uint32_t gchunk_pages,
                                                                uint32_t max_gchunks,
                                                                uint32_t chunk_pages)
{
    AttnSeqShape sh;
    sh.bad_len = L < 0 || (uint32_t)L > max_seq_len || (uint32_t)L > max_pages * 16u;
    sh.n_pages = sh.bad_len ? 0 : (L + 15) >> 4;
    sh.bad_skip = skip_raw > (uint32_t)sh.n_pages || skip_raw > max_gchunks * gchunk_pages;
    sh.skip = sh.bad_skip ? 0 : (int)skip_raw;
    const int cp = (int)chunk_pages;
    sh.n_g = (uint32_t)((sh.skip + (int)gchunk_pages - 1) / (int)gchunk_pages);
    const int own = (sh.n_pages - sh.skip + cp - 1) / cp;
    sh.n_chunks = sh.n_pages ? (own > 0 ? own : (sh.n_g ? 1 : 0)) : 0;
    return sh;
}

// Maximum that is NaN when either operand is NaN (the chunk maxima a logits
// producer hands to the sampler flag NaN this way).
__device__ __forceinline__ float nan_max(float x, float y)
{
    float r;
    asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(x), "f"(y));
    return r;
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi)
{
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t *>(&v);
}

// Two-term bf16 split of a pair: (a, b) ~= hi + lo with hi = RN(a, b) and
// lo = RN of the residual, so a product against bf16 operands accumulated
// as hi.V + lo.V keeps about 16 mantissa bits of a and b instead of 8.
__device__ __forceinline__ void split_bf16x2(float a, float b, uint32_t &hi, uint32_t &lo)
{
    hi = pack_bf16x2(a, b);
    lo = pack_bf16x2(a - __uint_as_float(hi << 16), b - __uint_as_float(hi & 0xFFFF0000u));
}

// Philox4x32-10 (Salmon et al., SC'11).
__host__ __device__ __forceinline__ void philox4x32_10(uint32_t c0, uint32_t c1, uint32_t c2,
                                                       uint32_t c3, uint32_t k0, uint32_t k1,
                                                       uint32_t (&out)[4])
{
#pragma unroll
    for (int r = 0; r < 10; r++) {
#if defined(__CUDA_ARCH__)
        const uint32_t lo0 = 0xD2511F53u * c0, hi0 = __umulhi(0xD2511F53u, c0);
        const uint32_t lo1 = 0xCD9E8D57u * c2, hi1 = __umulhi(0xCD9E8D57u, c2);
#else
        const uint64_t p0 = (uint64_t)0xD2511F53u * c0, p1 = (uint64_t)0xCD9E8D57u * c2;
        const uint32_t lo0 = (uint32_t)p0, hi0 = (uint32_t)(p0 >> 32);
        const uint32_t lo1 = (uint32_t)p1, hi1 = (uint32_t)(p1 >> 32);
#endif
        const uint32_t n0 = hi1 ^ c1 ^ k0, n2 = hi0 ^ c3 ^ k1;
        c0 = n0;
        c1 = lo1;
        c2 = n2;
        c3 = lo0;
        k0 += 0x9E3779B9u;
        k1 += 0xBB67AE85u;
    }
    out[0] = c0;
    out[1] = c1;
    out[2] = c2;
    out[3] = c3;
}

// Four N(0,1) samples from one Philox block by the Box-Muller transform
// (synthetic data only: the SFU approximations of log / sin / cos are used
// for speed; every consumer regenerates values with this same function).
__device__ __forceinline__ void philox_normal4(uint64_t seed, uint32_t c0, uint32_t c1,
                                               uint32_t c2, float (&z)[4], uint32_t c3 = 0u)
{
    uint32_t x[4];
    philox4x32_10(c0, c1, c2, c3, (uint32_t)seed, (uint32_t)(seed >> 32), x);
#pragma unroll
    for (int k = 0; k < 2; k++) {
        const float u1 = ((float)((x[2 * k] >> 8) + 1u)) * (1.0f / 16777216.0f);
        const float u2 = ((float)(x[2 * k + 1] >> 8)) * (1.0f / 16777216.0f);
        const float rad = __fsqrt_rn(-2.0f * __logf(u1));
        float s, c;
        __sincosf(6.283185307179586f * u2, &s, &c);
        z[2 * k] = rad * c;
        z[2 * k + 1] = rad * s;
    }
}

// -------------------------------------------------------------------- host
void set_error(const char *fmt, ...);
int cuda_fail(cudaError_t e, const char *what);  // records and returns RT_ECUDA
int num_sms();
// Encode a 2-D bf16 tensor map over rows of 128 elements (256 B), box
// 64 x 16 with 128-byte swizzle.  Returns 0 or RT_* error.
int encode_kv_rows_map(CUtensorMap *map, const void *base, uint64_t rows);
// 2-D map over a row-major bf16 matrix [rows][k] (k contiguous), box of
// box_k (64 or 32) columns x box_rows rows with 128- or 64-byte swizzle: the
// K-major operand tile of a tcgen05 MMA.  Out-of-range rows and columns
// read zero.
int encode_bf16_kmajor_map(CUtensorMap *map, const void *base, uint64_t k, uint64_t rows,
                           uint64_t row_stride_bytes, uint32_t box_rows, uint32_t box_k);
// 2-D map over a row-major fp32 matrix [rows][cols] for TMA stores: box of
// 32 columns (128 bytes) x box_rows rows, 128-byte swizzle.  Stores are
// clipped at the matrix edge.
int encode_f32_store_map(CUtensorMap *map, const void *base, uint64_t cols, uint64_t rows,
                         uint64_t row_stride_bytes, uint32_t box_rows);

}  // namespace rt
