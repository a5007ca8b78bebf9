// rt_host.cu - host-side plumbing of the C ABI: per-thread error text,
// device queries, tensor-map encoding through the driver entry point, and
// the synthetic-data fill kernels.
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "rlrt.h"
#include "rt_common.cuh"

namespace rt {

static thread_local char g_err[512];

void set_error(const char *fmt, ...)
{
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof(g_err), fmt, ap);
    va_end(ap);
}

int cuda_fail(cudaError_t e, const char *what)
{
    set_error("%s: %s (%d)", what, cudaGetErrorString(e), (int)e);
    return RT_ECUDA;
}

int num_sms()
{
    int dev = 0, n = 0;
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
        (void)cudaGetLastError();
        return 148;
    }
    return n;
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                  const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                  const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn()
{
    static std::once_flag once;
    static EncodeTiledFn fn = nullptr;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
        else
            (void)cudaGetLastError();
    });
    return fn;
}

int encode_kv_rows_map(CUtensorMap *map, const void *base, uint64_t rows)
{
    EncodeTiledFn fn = encode_fn();
    if (!fn) {
        set_error("cuTensorMapEncodeTiled unavailable from the driver");
        return RT_ECUDA;
    }
    if (((uintptr_t)base & 15u) != 0u || rows == 0 || rows > (1ull << 31)) {
        set_error("KV arena base must be 16-byte aligned and hold 1..2^31 rows (rows=%llu)",
                  (unsigned long long)rows);
        return RT_EINVAL;
    }
    cuuint64_t gdim[2] = {128u, (cuuint64_t)rows};
    cuuint64_t gstride[1] = {256u};
    cuuint32_t box[2] = {64u, 16u};
    cuuint32_t estride[2] = {1u, 1u};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(base), gdim,
                    gstride, box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        set_error("cuTensorMapEncodeTiled failed (CUresult %d)", (int)r);
        return RT_ECUDA;
    }
    return RT_OK;
}

int encode_bf16_kmajor_map(CUtensorMap *map, const void *base, uint64_t k, uint64_t rows,
                           uint64_t row_stride_bytes, uint32_t box_rows, uint32_t box_k)
{
    EncodeTiledFn fn = encode_fn();
    if (!fn) {
        set_error("cuTensorMapEncodeTiled unavailable from the driver");
        return RT_ECUDA;
    }
    if (((uintptr_t)base & 15u) != 0u || (row_stride_bytes & 15u) != 0u || k == 0 || rows == 0 ||
        box_rows == 0 || box_rows > 256u) {
        set_error("bf16 operand: base and row stride must be 16-byte aligned, box rows 1..256");
        return RT_EINVAL;
    }
    if (box_k != 64u && box_k != 32u) {
        set_error("bf16 operand: K box of 32 or 64 elements");
        return RT_EINVAL;
    }
    cuuint64_t gdim[2] = {(cuuint64_t)k, (cuuint64_t)rows};
    cuuint64_t gstride[1] = {(cuuint64_t)row_stride_bytes};
    cuuint32_t box[2] = {box_k, box_rows};
    cuuint32_t estride[2] = {1u, 1u};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(base), gdim,
                    gstride, box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    box_k == 64u ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        set_error("cuTensorMapEncodeTiled failed (CUresult %d)", (int)r);
        return RT_ECUDA;
    }
    return RT_OK;
}

int encode_f32_store_map(CUtensorMap *map, const void *base, uint64_t cols, uint64_t rows,
                         uint64_t row_stride_bytes, uint32_t box_rows)
{
    EncodeTiledFn fn = encode_fn();
    if (!fn) {
        set_error("cuTensorMapEncodeTiled unavailable from the driver");
        return RT_ECUDA;
    }
    if (((uintptr_t)base & 15u) != 0u || (row_stride_bytes & 15u) != 0u || cols == 0 ||
        rows == 0 || box_rows == 0 || box_rows > 256u) {
        set_error("fp32 output: base and row stride must be 16-byte aligned, box rows 1..256");
        return RT_EINVAL;
    }
    cuuint64_t gdim[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t gstride[1] = {(cuuint64_t)row_stride_bytes};
    cuuint32_t box[2] = {32u, box_rows};
    cuuint32_t estride[2] = {1u, 1u};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void *>(base), gdim,
                    gstride, box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        set_error("cuTensorMapEncodeTiled failed (CUresult %d)", (int)r);
        return RT_ECUDA;
    }
    return RT_OK;
}

}  // namespace rt

// ------------------------------------------------------------ fill kernels
namespace {

template <typename T>
__global__ void fill_normal_kernel(T *dst, uint64_t n, uint64_t seed, uint32_t stream, float mean,
                                   float stdv)
{
    const uint64_t groups = (n + 3u) / 4u;
    for (uint64_t g = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; g < groups;
         g += (uint64_t)gridDim.x * blockDim.x) {
        float z[4];
        rt::philox_normal4(seed, (uint32_t)g, (uint32_t)(g >> 32), stream, z);
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const uint64_t i = g * 4u + (uint64_t)k;
            if (i < n) {
                const float v = mean + stdv * z[k];
                if constexpr (sizeof(T) == 2)
                    dst[i] = __float2bfloat16_rn(v);
                else
                    dst[i] = v;
            }
        }
    }
}

template <typename T>
int launch_fill(T *dst, uint64_t n, uint64_t seed, uint32_t stream, float mean, float stdv,
                void *s)
{
    if (!dst && n) {
        rt::set_error("fill: null destination");
        return RT_EINVAL;
    }
    if (n == 0)
        return RT_OK;
    const uint64_t groups = (n + 3u) / 4u;
    uint64_t blocks = (groups + 255u) / 256u;
    const uint64_t cap = (uint64_t)rt::num_sms() * 16u;
    if (blocks > cap)
        blocks = cap;
    fill_normal_kernel<T><<<(unsigned)blocks, 256, 0, (cudaStream_t)s>>>(dst, n, seed, stream,
                                                                          mean, stdv);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? RT_OK : rt::cuda_fail(e, "fill_normal launch");
}

}  // namespace

extern "C" const char *rt_last_error(void) { return rt::g_err; }

extern "C" const char *rt_version(void) { return "rlrt-b200 0.1 sm_100a"; }

extern "C" int rt_fill_normal_bf16(void *dst, uint64_t n, uint64_t seed, uint32_t stream,
                                   float mean, float stdv, void *s)
{
    return launch_fill(reinterpret_cast<__nv_bfloat16 *>(dst), n, seed, stream, mean, stdv, s);
}

extern "C" int rt_fill_normal_f32(float *dst, uint64_t n, uint64_t seed, uint32_t stream,
                                  float mean, float stdv, void *s)
{
    return launch_fill(dst, n, seed, stream, mean, stdv, s);
}
