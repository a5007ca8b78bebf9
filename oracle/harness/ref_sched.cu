// ref_sched.cu - GPU harness around the reference's own scheduler, reward
// and prefix-resolve kernels.  TEST INFRASTRUCTURE ONLY.
//
// Compiled by oracle/Makefile with the reference's include directory and
// oracle/ref_cu_atomic_shim.h force-included, and linked (relocatable device
// code) with the reference's cu/gpu_scheduler.cu, cu/reward.cu and
// cu/kv_prefix.cu, unmodified, into oracle/_ref/libref_cuda.so.
//
// The reference rollout_worker (cu/gpu_scheduler.cu:26-83) only returns when
// it consumes the request_id == UINT64_MAX sentinel, and spins without bound
// while its DoneRing is full (cu/gpu_scheduler.cu:70-71).  So it is launched
// here only on rings in device memory whose contents make it finish by
// construction, checked on the host before the launch:
//   - the RequestRing holds every record before the launch (no producer
//     runs meanwhile), fewer than REQUEST_RING_SIZE of them, and the last is
//     the sentinel, so every pass consumes one record and pass n + 1 returns;
//   - the DoneRing starts empty and the requests before the sentinel are
//     fewer than its REQUEST_RING_SIZE slots, so no push ever finds it full.
#include <stdint.h>
#include <string.h>

#include "kv_prefix.h"  // the reference's headers
#include "reward.h"

__global__ void rollout_worker(RequestRing *, DoneRing *, GpuRolloutState *, uint64_t *);
__global__ void reward_score_kernel(RewardDesc *descs, int n, float *scores);
__global__ void kv_branch_resolve(KVPrefixTable *t, uint32_t *branch_ids, int64_t *out_offsets,
                                  int n);

// Returns 0, -1 when the rings could end in an endless wait (not launched),
// or a CUDA error code.
extern "C" int hx_ref_rollout_worker(RequestRing *req_d, DoneRing *done_d, GpuRolloutState *st_d,
                                     uint64_t *steps_d)
{
    static RequestRing rq;
    static DoneRing dn;
    cudaError_t e = cudaMemcpy(&rq, req_d, sizeof(rq), cudaMemcpyDeviceToHost);
    if (e == cudaSuccess)
        e = cudaMemcpy(&dn, done_d, sizeof(dn), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess)
        return (int)e;
    const uint32_t head = rq.cons.head, tail = rq.prod.tail;
    const uint32_t n = tail - head;
    if (head != 0u || n == 0u || n >= REQUEST_RING_SIZE)
        return -1;
    if (rq.slots[(tail - 1u) & (REQUEST_RING_SIZE - 1)].request_id != UINT64_MAX)
        return -1;
    if (dn.cons.head != 0u || dn.prod.tail != 0u)
        return -1;
    rollout_worker<<<1, 32>>>(req_d, done_d, st_d, steps_d);
    e = cudaDeviceSynchronize();
    return e == cudaSuccess ? 0 : (int)e;
}

extern "C" int hx_ref_reward_score(RewardDesc *descs_d, int n, float *scores_d)
{
    if (n <= 0)
        return 0;
    reward_score_kernel<<<(n + 255) / 256, 256>>>(descs_d, n, scores_d);
    const cudaError_t e = cudaDeviceSynchronize();
    return e == cudaSuccess ? 0 : (int)e;
}

extern "C" int hx_ref_kv_branch_resolve(KVPrefixTable *t_d, uint32_t *ids_d, int64_t *out_d, int n)
{
    if (n <= 0)
        return 0;
    kv_branch_resolve<<<(n + 255) / 256, 256>>>(t_d, ids_d, out_d, n);
    const cudaError_t e = cudaDeviceSynchronize();
    return e == cudaSuccess ? 0 : (int)e;
}

extern "C" uint64_t hx_ref_sizeof(int what)
{
    switch (what) {
    case 0: return sizeof(RequestRing);
    case 1: return sizeof(DoneRing);
    case 2: return sizeof(GpuRolloutState);
    case 3: return sizeof(KVPrefixTable);
    case 4: return sizeof(RewardDesc);
    default: return 0;
    }
}
