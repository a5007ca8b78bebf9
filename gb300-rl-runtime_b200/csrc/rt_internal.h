// rt_internal.h - cross-file hooks inside librlrt_b200.so (not exported).
#pragma once
#include <cuda_runtime.h>

#include "rlrt.h"

namespace rt {
// Set kernel attributes of the attention launch for these params so a later
// launch (e.g. inside stream capture) issues no attribute calls.
int attn_prepare(const rt_attn_params_t *p);
// Same for the tensor-core GEMM (its shared-memory opt-in on this device).
int gemm_prepare();
// rt_sample_rows with an optional programmatic dependent launch (the kernel
// waits for the previous kernel of the stream before reading the logits)
// and optional producer chunk maxima (rt_sample_rows_cmax).
int sample_rows_launch(const rt_sample_params_t *p, const float *logits,
                       const rt_sample_row_t *rows, uint32_t *tokens_out, cudaStream_t stream,
                       bool pdl, const float *cmax = nullptr, uint32_t cmax_stride = 0);
}  // namespace rt
