// ref_sample.cu - GPU harness around the reference's own sampler.
// TEST INFRASTRUCTURE ONLY.
//
// Compiled by oracle/Makefile with the reference's include directory and
// linked (relocatable device code) with the reference's cu/sample.cu,
// unmodified, into oracle/_ref/libref_cuda.so.  One thread per row runs the
// reference sample_token() on a private copy of that row's logits.
//
// The reference draws its uniform from xoshiro256** state
// (cu/sample.cu:92,114: xoshiro256_next(st->rng_state) & 0x00FFFFFF).  The
// first output of xoshiro256** depends only on state word 1
// (result = rotl(s1 * 5, 7) * 9), which is invertible, so the caller passes
// s1 chosen to make that first draw equal the Philox uniform the B200
// sampler uses; no reference source is patched.
#include <stdint.h>

#include "sample.h"  // the reference's header

__global__ void hx_ref_sample_kernel(float *logits, uint32_t vocab, uint64_t stride,
                                     const float *temperature, const uint16_t *top_k,
                                     const float *top_p, const uint64_t *s1, uint32_t *out,
                                     uint32_t rows)
{
    const uint32_t r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= rows)
        return;
    SampleState st;
    st.rng_state[0] = 0x0123456789abcdefULL;
    st.rng_state[1] = s1[r];
    st.rng_state[2] = 0xfedcba9876543210ULL;
    st.rng_state[3] = 0x0f0f0f0f0f0f0f0fULL;
    st.temperature = temperature[r];
    st.top_k = top_k[r];
    st.top_p = top_p[r];
    st.vocab_size = vocab;
    out[r] = sample_token(&st, logits + (uint64_t)r * stride);
}

extern "C" int hx_ref_sample_rows(float *logits, uint32_t vocab, uint64_t stride,
                                  const float *temperature, const uint16_t *top_k,
                                  const float *top_p, const uint64_t *s1, uint32_t *out,
                                  uint32_t rows)
{
    // the reference keeps a 256-entry threshold array per thread
    cudaDeviceSetLimit(cudaLimitStackSize, 4096);
    hx_ref_sample_kernel<<<(rows + 31) / 32, 32>>>(logits, vocab, stride, temperature, top_k,
                                                   top_p, s1, out, rows);
    cudaError_t e = cudaDeviceSynchronize();
    return e == cudaSuccess ? 0 : (int)e;
}
