// The cross-attention keys and values of a sequence start, on the tcgen05
// tensor cores: recordSequenceStart (Lib/WhisperEACP/Decoder/Decoder.cpp:
// 121-146) for every window of a batch in one launch.
//
// For window b, layer l and head h the cache block [X][K_h | V_h] is
// E_b . [Wk_h ; Wv_h]^T: the encoder rows (fp32) against the head's D key
// rows then its D value rows of k_proj / v_proj.  Stacking every (layer,
// head) group's 2D weight rows gives one product per window,
// E_b [X, d] x W^T [d, L*2d], whose columns are the groups' blocks side by
// side; the kernel writes each 2D-column slice straight into the group's
// block of the cache layout [layer][window][head][X][K | V] (a layer's keys
// and values for every window contiguous, as one step's cross attention of
// that layer reads them; 64-wide heads:
// with each 256-byte row's 16-byte pieces rotated by cross_piece, the order
// the decode kernel's tensor-core attention reads).  The value bias is not
// added here: the attention adds it after normalising (the weights sum to
// one).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace wsp {

// Weight rows of a weight tile (the MMA's N) and k columns of a block.
constexpr int kCrossTileRows = 256;
constexpr int kCrossBlockCols = 64;

// Element offset of (weight row n, column k) in the cross projection's
// tensor-core layout: tiles of 256 weight rows, each kblocks blocks of 64
// columns (128 bytes a row, 32 KB a block), the 16-byte pieces of row n
// rotated by n % 8 (the 128-byte swizzle of the shared-memory descriptor).
// A (tile, block) is one contiguous 32 KB copy.
__host__ __device__ inline size_t cross_weight_offset(int n, int k, int kblocks) {
    const int tile = n / kCrossTileRows, r = n % kCrossTileRows, kb = k / kCrossBlockCols, c = (k / 8) % 8;
    return (((size_t)tile * kblocks + kb) * kCrossTileRows + r) * kCrossBlockCols + ((c ^ (r % 8)) * 8) + k % 8;
}

struct CrossKvArgs {
    const float* encoder;   // fp32 [windows][row_stride][width], 16-byte aligned
    const void* weight;     // 16-bit, cross_weight_offset layout, n_tiles x kblocks blocks
    void* out;              // 16-bit [layers][windows][heads][row_stride][2 * head_width]
    int windows;
    int rows;               // encoder rows of each window projected (<= row_stride)
    int row_stride;         // rows a window holds in `encoder` and in `out` (X)
    int width;              // d: the product's inner size (a multiple of 4)
    int kblocks;            // ceil(d / 64)
    int columns;            // L * 2d: weight rows
    int head_width;         // D
    int groups;             // L * H
    int heads;              // H
    int* status;            // nonzero on return: a bounded wait gave up (which one)
    // The linear form (the encoder's products): with linear_out set, the
    // product of `windows` (1) x `rows` rows is written row-major to
    // linear_out [rows][columns] as gelu?(acc + bias[n]) (+ residual[row][n]
    // when residual is set, which may be linear_out itself) instead of into
    // the cross cache; head_width, groups and heads are then unused.
    float* linear_out;
    const float* bias;
    const float* residual;
    int gelu;
};

// Shared memory one CTA of the kernel asks for.
size_t cross_kv_shared_bytes();

// One launch over every window (or the linear form's rows): persistent, at
// most one CTA per SM.
// half: fp16 storage (else bf16).  Throws std::runtime_error on a launch
// failure.
void launch_cross_kv(bool half, const CrossKvArgs& args, int sm_count, cudaStream_t stream);

}  // namespace wsp
