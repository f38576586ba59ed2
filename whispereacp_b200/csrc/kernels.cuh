// Kernels outside the decode step: the standalone masked argmax.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace wsp {

enum class Storage : int { f16 = 1, bf16 = 2 };

inline int padded(int k) { return (k + 31) / 32 * 32; }

// The fold of per-group (value, index) candidates of each row into its id.
struct ArgmaxFinalArgs {
    const float* candidate_values;
    const uint32_t* candidate_indices;
    int candidates;          // per row
    int rows;
    int rows_per_window;     // unused by the standalone argmax (1)
    int step_tokens;
    uint32_t* row_tokens;    // [rows]
    uint32_t* ring;          // unused by the standalone argmax (null)
    int ring_stride;
    const int* position;
};

// Standalone masked argmax over [rows, length] fp32 logits (Argmax.h:207-262).
void launch_argmax_rows(const float* logits, const float* mask, uint32_t* out, int rows,
                        int length, float* candidate_values, uint32_t* candidate_indices,
                        int groups_per_row, cudaStream_t stream);
int argmax_groups_per_row(int length);

// The fixed scratch of wsp_argmax_no_alloc: room for this many per-group
// (value, index) candidate pairs, rows x argmax_groups_per_row(length).
constexpr int kNoAllocArgmaxCandidates = 65536;

// This device's address of that scratch (kNoAllocArgmaxCandidates floats,
// then as many uint32 indices), looked up with cudaGetSymbolAddress the first
// time a device asks, with that device current, and remembered after.
cudaError_t no_alloc_argmax_scratch(int device, void** scratch);

}  // namespace wsp
