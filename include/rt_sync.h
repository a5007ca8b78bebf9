/*
 * rt_sync.h - memory-ordering primitives shared by host C and device CUDA.
 *
 * Every ring in this runtime lives in pinned, mapped host memory
 * (cudaHostAllocMapped) so that a host thread and a GPU kernel can be the
 * two ends of one single-producer/single-consumer queue.  The two sides
 * therefore need acquire/release operations that are valid at *system*
 * scope: on the host they are the compiler's __atomic builtins, on the
 * device they are ld.acquire.sys / st.release.sys PTX instructions.
 *
 * This header replaces the reference's use of C11 <stdatomic.h> calls on
 * volatile fields (reference include/ring.h:40-67, include/completion.h:65-85,
 * include/request.h:88-149), which do not compile as device code.
 */
#pragma once
#include <stdint.h>

#if defined(__CUDACC__)
#define RT_HD __host__ __device__
#else
#define RT_HD
#endif

#if defined(__cplusplus)
#define RT_STATIC_ASSERT(c, m) static_assert(c, m)
#else
#define RT_STATIC_ASSERT(c, m) _Static_assert(c, m)
#endif

static inline RT_HD uint32_t
rt_load_acquire_u32(const volatile uint32_t *p)
{
#if defined(__CUDA_ARCH__)
    uint32_t v;
    asm volatile("ld.acquire.sys.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
#else
    return __atomic_load_n(p, __ATOMIC_ACQUIRE);
#endif
}

static inline RT_HD uint32_t
rt_load_relaxed_u32(const volatile uint32_t *p)
{
#if defined(__CUDA_ARCH__)
    uint32_t v;
    asm volatile("ld.relaxed.sys.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
#else
    return __atomic_load_n(p, __ATOMIC_RELAXED);
#endif
}

static inline RT_HD void
rt_store_release_u32(volatile uint32_t *p, uint32_t v)
{
#if defined(__CUDA_ARCH__)
    asm volatile("st.release.sys.u32 [%0], %1;" :: "l"(p), "r"(v) : "memory");
#else
    __atomic_store_n(p, v, __ATOMIC_RELEASE);
#endif
}

/* Relaxed counter bump (overflow counters).  System scope on the device so
 * that a counter in mapped host memory is updated atomically w.r.t. the CPU. */
static inline RT_HD void
rt_count_u32(volatile uint32_t *p)
{
#if defined(__CUDA_ARCH__)
    atomicAdd_system((unsigned int *)p, 1u);
#else
    __atomic_add_fetch((uint32_t *)p, 1u, __ATOMIC_RELAXED);
#endif
}

/* Copy of one packed ring record.  Packed structs such as the 34-byte
 * RolloutRequest sit at unaligned addresses, so the copy assumes no
 * alignment beyond one byte.  On the host it is a plain memcpy: the ring
 * index load before it (acquire) or the index store after it (release)
 * orders it, so the record needs no volatile access of its own, and the
 * compiler may move it in whole words.  On the device (only the done-ring
 * slow path copies records this way) it stays a byte loop of volatile
 * accesses to the mapped host memory. */
static inline RT_HD void
rt_copy_bytes(void *dst, const volatile void *src, uint32_t n)
{
#if defined(__CUDA_ARCH__)
    const volatile uint8_t *s = (const volatile uint8_t *)src;
    uint8_t *d = (uint8_t *)dst;
    for (uint32_t i = 0; i < n; i++)
        d[i] = s[i];
#else
    __builtin_memcpy(dst, (const void *)src, n);
#endif
}
