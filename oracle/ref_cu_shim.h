/* Force-included when compiling the reference's CUDA sources
 * (oracle/Makefile, _ref/libref_cuda.so).  As shipped they do not compile
 * with nvcc: headers compiled as C++ use C11 _Static_assert, the step calls
 * __sync_warp() (CUDA's intrinsic is __syncwarp), uses CUDART_INF_F without
 * including math_constants.h, and calls kv_layout.h's host-only static
 * inline helpers from device code.  These spellings are mapped to CUDA's
 * own (kv_layout.h is read once here with its helpers marked host+device);
 * the reference files are not touched. */
#pragma once
#include <stddef.h>
#include <stdint.h>
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <math_constants.h>
#define _Static_assert(cond, msg) static_assert(cond, msg)
#define __sync_warp() __syncwarp()
#define inline __host__ __device__ inline
#include "kv_layout.h"
#undef inline
