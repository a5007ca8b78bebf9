// kv_prefix.cu - device-side branch resolution over the copy-on-write prefix
// table (reference cu/kv_prefix.cu:4-23, kv_branch_resolve and
// d_kv_branch_total_offset).
//
// The table is the host's KVPrefixTable (kv_prefix.h), copied to device
// memory or mapped, byte for byte.  Its records are packed (28 and 36
// bytes), so the 64-bit offsets sit on 4-byte boundaries and are read as
// two 32-bit words.  One thread resolves one branch id; the kernel is a
// handful of dependent loads per id, latency-bound for any realistic n.
#include <cstddef>
#include <cstdint>

#include "kv_prefix.h"
#include "rlrt.h"
#include "rt_common.cuh"

namespace {

static_assert(offsetof(KVPrefixTable, branches) % 4 == 0, "branch records start 4-byte aligned");
static_assert(offsetof(KVPrefix, refcnt) == 4 && offsetof(KVPrefix, kv_block_offset) == 8,
              "KVPrefix layout");
static_assert(offsetof(KVBranch, prefix_id) == 8 && offsetof(KVBranch, delta_kv_offset) == 12,
              "KVBranch layout");

__device__ __forceinline__ int64_t ld_i64_w4(const void *p)
{
    const uint32_t *w = static_cast<const uint32_t *>(p);
    return (int64_t)(((uint64_t)__ldg(w + 1) << 32) | (uint64_t)__ldg(w));
}

// Reference semantics (cu/kv_prefix.cu:4-15): an id past MAX_BRANCHES gives
// -1; a branch whose prefix id is out of range, or whose prefix has no
// references left, resolves to its own delta offset; otherwise to the
// prefix's kv_block_offset.  (The host kv_branch_total_offset differs: it
// returns the prefix's offset, -1 after release, whatever the refcount.)
__global__ void __launch_bounds__(256)
kv_branch_resolve_kernel(const KVPrefixTable *t, const uint32_t *ids, int64_t *out, uint32_t n)
{
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n)
        return;
    const uint32_t id = __ldg(ids + i);
    int64_t r = -1;
    if (id < MAX_BRANCHES) {
        const KVBranch *b = &t->branches[id];
        const uint32_t pid = __ldg(reinterpret_cast<const uint32_t *>(b) + 2);
        const int64_t delta = ld_i64_w4(reinterpret_cast<const uint32_t *>(b) + 3);
        r = delta;
        if (pid < MAX_PREFIXES) {
            const KVPrefix *p = &t->prefixes[pid];
            if (__ldg(reinterpret_cast<const uint32_t *>(p) + 1) != 0u)
                r = ld_i64_w4(reinterpret_cast<const uint32_t *>(p) + 2);
        }
    }
    out[i] = r;
}

}  // namespace

extern "C" int rt_kv_branch_resolve(const KVPrefixTable *table, const uint32_t *branch_ids,
                                    int64_t *out_offsets, uint32_t n, void *stream)
{
    if (n == 0)
        return RT_OK;
    if (!table || !branch_ids || !out_offsets) {
        rt::set_error("kv_branch_resolve: null table, ids or output");
        return RT_EINVAL;
    }
    if ((reinterpret_cast<uintptr_t>(table) & 7u) || (reinterpret_cast<uintptr_t>(out_offsets) & 7u) ||
        (reinterpret_cast<uintptr_t>(branch_ids) & 3u)) {
        rt::set_error("kv_branch_resolve: misaligned table, ids or output");
        return RT_EINVAL;
    }
    kv_branch_resolve_kernel<<<(n + 255u) / 256u, 256, 0, (cudaStream_t)stream>>>(
        table, branch_ids, out_offsets, n);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? RT_OK : rt::cuda_fail(e, "kv_branch_resolve: launch");
}
