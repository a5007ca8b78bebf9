// ref_fixed128.cu - GPU harness around the reference's own fixed128 decode
// step.  TEST INFRASTRUCTURE ONLY.
//
// Compiled by oracle/Makefile with the reference's include directory and
// linked (relocatable device code) with the reference's
// cu/attention_decode.cu and cu/prefetch.cu, unmodified, into
// oracle/_ref/libref_cuda.so.  One 32-thread block per descriptor calls
// attention_decode_step_fixed128 exactly as the reference's
// process_descriptor does (cu/worker.cu:30-51: the block's address from
// the arena, slot = output_token_offset & (io_slots - 1), seq_len =
// num_kv_blocks or 1), except that each descriptor's output row goes to
// its own o_out[i] so the rows of descriptors sharing a slot stay apart.
//
// Bounds (checked by the caller): every kv_block_offset < n_blocks, and
// the step reads the full 16 KiB block (prefetch_issue), so the arena
// holds n_blocks whole blocks of block_size >= 16 KiB; slot < io_slots
// rows of q (or q == NULL); 16 KiB of dynamic shared memory per block (the
// step stages one block into stage 0 only).
#include <stdint.h>

#include "attention_decode.h"  // the reference's header
#include "descriptor.h"

__global__ void hx_ref_fixed128_kernel(const Descriptor *descs, uint32_t n, const uint8_t *arena,
                                       uint64_t block_size, SampleState *sample_st,
                                       const __half *q_buffer, uint32_t io_slots, float *o_out,
                                       uint32_t *token, uint32_t *bytes, uint32_t *tiles,
                                       uint64_t *cycles)
{
    extern __shared__ uint8_t smem[];
    const uint32_t i = blockIdx.x;
    if (i >= n)
        return;
    const Descriptor desc = descs[i];
    const uint32_t slot = io_slots == 0 ? 0U : (desc.output_token_offset & (io_slots - 1U));
    DecodeStepArgs args;
    args.q_ptr = q_buffer ? (const void *)(q_buffer + slot * DECODE_FIXED_HEAD_DIM) : NULL;
    args.o_ptr = (void *)(o_out + (uint64_t)i * DECODE_FIXED_HEAD_DIM);
    args.seq_len = desc.num_kv_blocks == 0 ? 1U : (uint32_t)desc.num_kv_blocks;
    args.head_dim = DECODE_FIXED_HEAD_DIM;
    args.kv_block_base_idx = desc.kv_block_offset;
    args.kv_block_count = 1;
    args.output_token_offset = slot;
    const uint8_t *kv = arena + (uint64_t)desc.kv_block_offset * block_size;
    DecodeStepResult r = attention_decode_step_fixed128(&desc, &args, kv, sample_st, smem);
    if ((threadIdx.x & 31U) == 0) {
        token[i] = r.token_id;
        bytes[i] = r.bytes_touched;
        tiles[i] = r.tile_count;
        cycles[i] = r.cycle_estimate;
    }
}

extern "C" int hx_ref_fixed128(const Descriptor *descs, uint32_t n, const uint8_t *arena,
                               uint64_t block_size, SampleState *sample_st,
                               const __half *q_buffer, uint32_t io_slots, float *o_out,
                               uint32_t *token, uint32_t *bytes, uint32_t *tiles, uint64_t *cycles)
{
    if (n == 0)
        return 0;
    hx_ref_fixed128_kernel<<<n, 32, 16384>>>(descs, n, arena, block_size, sample_st, q_buffer,
                                             io_slots, o_out, token, bytes, tiles, cycles);
    cudaError_t e = cudaDeviceSynchronize();
    return e == cudaSuccess ? 0 : (int)e;
}
