// rt_internal.h - cross-file hooks inside librlrt_b200.so (not exported).
#pragma once
#include <cuda_runtime.h>

#include "rlrt.h"

namespace rt {
// Set kernel attributes of the attention launch for these params so a later
// launch (e.g. inside stream capture) issues no attribute calls.
int attn_prepare(const rt_attn_params_t *p);
// Paged decode attention (grouped when gp is not null) with an optional
// device word holding this launch's largest per-sequence chunk count
// (rt::attn_seq_shape over the launch's lengths and skips, at least 1); the
// kernel then hands out no chunks past it.
int attn_launch(const rt_attn_params_t *p, const rt_attn_group_params_t *gp, const void *q,
                const void *kv_arena, const int32_t *page_table, const int32_t *seq_lens,
                const rt_attn_group_t *groups, const uint32_t *n_groups,
                const uint32_t *skip_pages, float *out, void *workspace,
                size_t workspace_bytes, const uint32_t *dyn_chunks, cudaStream_t stream);
// The plan's item shape for these params: chunk pages of the sequence items,
// and of the group items with their count (1 and 0 without groups).
int attn_item_shape(const rt_attn_params_t *p, const rt_attn_group_params_t *gp,
                    uint32_t *chunk_pages, uint32_t *gchunk_pages, uint32_t *max_gchunks);
// Same for the tensor-core GEMM (its shared-memory opt-in on this device).
int gemm_prepare();
// rt_sample_rows with an optional programmatic dependent launch (the kernel
// waits for the previous kernel of the stream before reading the logits)
// and optional producer chunk maxima (rt_sample_rows_cmax).
int sample_rows_launch(const rt_sample_params_t *p, const float *logits,
                       const rt_sample_row_t *rows, uint32_t *tokens_out, cudaStream_t stream,
                       bool pdl, const float *cmax = nullptr, uint32_t cmax_stride = 0);
}  // namespace rt
