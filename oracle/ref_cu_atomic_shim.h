/* Force-included when compiling the reference's cu/gpu_scheduler.cu,
 * cu/reward.cu and cu/kv_prefix.cu and their harness (oracle/Makefile,
 * _ref/libref_cuda.so).  TEST INFRASTRUCTURE ONLY.
 *
 * As shipped these do not compile with nvcc:
 *  - include/request.h uses C11 <stdatomic.h> (atomic_load_explicit /
 *    atomic_store_explicit on volatile uint32_t ring indices) from device
 *    code, which C++ cannot compile.  GCC's header is kept out (its include
 *    guard is defined first) and the two calls are provided here as
 *    system-scope cuda::atomic_ref operations with the same memory orders:
 *    the rings are shared between host and device.
 *  - request.h's done_ring_push (device) calls the host-only static inline
 *    done_ring_record_overflow; request.h is read once here with its
 *    static inline helpers marked host+device.
 *  - headers compiled as C++ use C11 _Static_assert; it maps to
 *    static_assert, except where REF_SHIM_NO_STATIC_ASSERT is defined:
 *    include/kv_prefix.h asserts packed sizes 24 and 28 for records that are
 *    28 and 36 bytes, so cu/kv_prefix.cu is compiled with the assertions
 *    off, as the reference's own C build of src/kv_prefix.c needs.
 * No reference file is edited. */
#pragma once
#include <stddef.h>
#include <stdint.h>
#include <cuda_runtime.h>
#include <cuda/atomic>

#ifdef REF_SHIM_NO_STATIC_ASSERT
#define _Static_assert(cond, msg)
#else
#define _Static_assert(cond, msg) static_assert(cond, msg)
#endif

#define _STDATOMIC_H 1
#define memory_order_relaxed cuda::std::memory_order_relaxed
#define memory_order_acquire cuda::std::memory_order_acquire
#define memory_order_release cuda::std::memory_order_release

template <class T>
__host__ __device__ inline T atomic_load_explicit(volatile T *p, cuda::std::memory_order mo)
{
    return cuda::atomic_ref<T, cuda::thread_scope_system>(*const_cast<T *>(p)).load(mo);
}

template <class T, class U>
__host__ __device__ inline void atomic_store_explicit(volatile T *p, U v, cuda::std::memory_order mo)
{
    cuda::atomic_ref<T, cuda::thread_scope_system>(*const_cast<T *>(p)).store((T)v, mo);
}

#define inline __host__ __device__ inline
#include "request.h"
#undef inline
