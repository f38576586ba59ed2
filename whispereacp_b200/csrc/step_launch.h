// Host entry points of the persistent decode kernel (step.cu).
#pragma once

#include "step.cuh"

namespace wsp {

// Input rows of a general product's tile in a launch with these parameters.
int decode_tile_rows(const StepParams& p);

// Shared memory the kernel needs besides its weight-stream ring (bytes).
size_t decode_work_bytes(bool half, const StepParams& p, int max_chunk);

// CTAs of the decode kernel one SM holds for these parameters (0: none fit).
int decode_blocks_per_sm(bool half, const StepParams& p, int max_chunk);

// One cooperative launch running p.steps steps of p.ops; max_chunk bounds the
// keys a cross-attention item holds in shared memory.
void launch_decode(bool half, const StepParams& p, int max_chunk, int grid, cudaStream_t stream);

}  // namespace wsp
