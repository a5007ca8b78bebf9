// reward.cu - reward scoring, group-normalised advantages, and the NCCL
// allgather of per-rollout rewards (the path's only cross-GPU exchange).
#include <chrono>
#include <cstdint>
#include <cstring>
#include <thread>

#include <nccl.h>

#include "reward.h"
#include "rlrt.h"
#include "rt_common.cuh"

namespace {

// reference cu/reward.cu:4-15
__global__ void reward_score_kernel(RewardDesc *descs, uint32_t n, float *scores)
{
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n)
        return;
    const float v = reward_score_mock_inline(descs[i].token_count);
    descs[i].reward = v;
    if (scores)
        scores[i] = v;
}

// One thread per group; explicit round-to-nearest operations fix the fp32
// operation order so the result is reproducible bit for bit.
__global__ void grpo_advantages_kernel(const float *r, uint32_t n_groups, uint32_t G, float eps,
                                       float *adv)
{
    const uint32_t g = blockIdx.x * blockDim.x + threadIdx.x;
    if (g >= n_groups)
        return;
    const float *x = r + (size_t)g * G;
    float sum = 0.0f;
    for (uint32_t i = 0; i < G; i++)
        sum = __fadd_rn(sum, x[i]);
    const float mean = __fdiv_rn(sum, (float)G);
    float var = 0.0f;
    for (uint32_t i = 0; i < G; i++) {
        const float d = __fsub_rn(x[i], mean);
        var = __fadd_rn(var, __fmul_rn(d, d));
    }
    const float den = __fadd_rn(__fsqrt_rn(__fdiv_rn(var, (float)G)), eps);
    for (uint32_t i = 0; i < G; i++)
        adv[(size_t)g * G + i] = __fdiv_rn(__fsub_rn(x[i], mean), den);
}

int nccl_fail(ncclResult_t r, const char *what)
{
    rt::set_error("%s: %s (%d)", what, ncclGetErrorString(r), (int)r);
    return RT_ECUDA;
}

}  // namespace

extern "C" int rt_reward_score(RewardDesc *descs, uint32_t n, float *scores, void *stream)
{
    if (!descs && n) {
        rt::set_error("reward_score: null descriptors");
        return RT_EINVAL;
    }
    if (n == 0)
        return RT_OK;
    reward_score_kernel<<<(n + 255u) / 256u, 256, 0, (cudaStream_t)stream>>>(descs, n, scores);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? RT_OK : rt::cuda_fail(e, "reward_score: launch");
}

extern "C" int rt_grpo_advantages(const float *rewards, uint32_t n, uint32_t G, float eps,
                                  float *adv, void *stream)
{
    if (!rewards || !adv || G == 0 || n % G) {
        rt::set_error("grpo_advantages: n (%u) must be a positive multiple of G (%u)", n, G);
        return RT_EINVAL;
    }
    const uint32_t groups = n / G;
    if (groups == 0)
        return RT_OK;
    grpo_advantages_kernel<<<(groups + 127u) / 128u, 128, 0, (cudaStream_t)stream>>>(
        rewards, groups, G, eps, adv);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? RT_OK : rt::cuda_fail(e, "grpo_advantages: launch");
}

extern "C" int rt_nccl_unique_id(void *id128)
{
    static_assert(sizeof(ncclUniqueId) == 128, "ncclUniqueId is 128 bytes");
    if (!id128) {
        rt::set_error("nccl_unique_id: null output");
        return RT_EINVAL;
    }
    ncclUniqueId id;
    ncclResult_t r = ncclGetUniqueId(&id);
    if (r != ncclSuccess)
        return nccl_fail(r, "ncclGetUniqueId");
    memcpy(id128, &id, sizeof(id));
    return RT_OK;
}

extern "C" int rt_nccl_init(void **comm, int nranks, const void *id128, int rank)
{
    if (!comm || !id128 || nranks < 1 || rank < 0 || rank >= nranks) {
        rt::set_error("nccl_init: bad arguments (rank %d of %d)", rank, nranks);
        return RT_EINVAL;
    }
    ncclUniqueId id;
    memcpy(&id, id128, sizeof(id));
    ncclComm_t c = nullptr;
    ncclResult_t r = ncclCommInitRank(&c, nranks, id, rank);
    if (r != ncclSuccess)
        return nccl_fail(r, "ncclCommInitRank");
    *comm = c;
    return RT_OK;
}

extern "C" int rt_nccl_destroy(void *comm)
{
    if (!comm)
        return RT_OK;
    ncclResult_t r = ncclCommDestroy(static_cast<ncclComm_t>(comm));
    return r == ncclSuccess ? RT_OK : nccl_fail(r, "ncclCommDestroy");
}

extern "C" int rt_reward_allgather(void *comm, const float *send, float *recv, uint64_t n_per_rank,
                                   void *stream)
{
    if (!comm || !send || !recv) {
        rt::set_error("reward_allgather: null argument");
        return RT_EINVAL;
    }
    ncclResult_t r = ncclAllGather(send, recv, n_per_rank, ncclFloat32,
                                   static_cast<ncclComm_t>(comm), (cudaStream_t)stream);
    return r == ncclSuccess ? RT_OK : nccl_fail(r, "ncclAllGather");
}

extern "C" int rt_nccl_wait(void *comm, void *stream, uint32_t timeout_ms)
{
    const auto t0 = std::chrono::steady_clock::now();
    for (;;) {
        cudaError_t q = cudaStreamQuery((cudaStream_t)stream);
        if (q == cudaSuccess)
            return RT_OK;
        if (q != cudaErrorNotReady)
            return rt::cuda_fail(q, "nccl_wait: stream");
        if (comm) {
            ncclResult_t async = ncclSuccess;
            ncclCommGetAsyncError(static_cast<ncclComm_t>(comm), &async);
            if (async != ncclSuccess && async != ncclInProgress) {
                ncclCommAbort(static_cast<ncclComm_t>(comm));
                return nccl_fail(async, "nccl_wait: communicator error (aborted)");
            }
        }
        const auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(
                            std::chrono::steady_clock::now() - t0).count();
        if ((uint64_t)ms > timeout_ms) {
            if (comm)
                ncclCommAbort(static_cast<ncclComm_t>(comm));
            rt::set_error("nccl_wait: no completion within %u ms; communicator aborted", timeout_ms);
            return RT_ETIMEOUT;
        }
        std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
}
