/*
 * mmio.h - doorbell store/load with the fences a device register needs.
 * Drop-in for reference include/mmio.h:5-34 (same three inline functions).
 * On a B200 host the doorbell is a word of mapped host memory that the
 * persistent GPU worker may poll; the store fence orders the descriptor
 * write before the doorbell value becomes visible.
 */
#pragma once
#include <stdint.h>

static inline void
mmio_wmb(void)
{
#if defined(__x86_64__)
    __asm__ volatile("sfence" ::: "memory");
#elif defined(__aarch64__)
    __asm__ volatile("dsb st" ::: "memory");
#else
    __sync_synchronize();
#endif
}

static inline void
mmio_write32(volatile uint32_t *addr, uint32_t value)
{
    mmio_wmb();
    *addr = value;
}

static inline uint32_t
mmio_read32(volatile uint32_t *addr)
{
    uint32_t v = *addr;
#if defined(__aarch64__)
    __asm__ volatile("dmb oshld" ::: "memory");
#else
    __asm__ volatile("" ::: "memory");
#endif
    return v;
}
