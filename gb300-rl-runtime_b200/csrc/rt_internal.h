// rt_internal.h - cross-file hooks inside librlrt_b200.so (not exported).
#pragma once
#include "rlrt.h"

namespace rt {
// Set kernel attributes of the attention launch for these params so a later
// launch (e.g. inside stream capture) issues no attribute calls.
int attn_prepare(const rt_attn_params_t *p);
// Same for the sampler (its shared-memory opt-in).
int sample_prepare();
}  // namespace rt
