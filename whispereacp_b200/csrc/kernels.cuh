// Kernel parameter blocks and launchers for one decoder step.
//
// A step of T tokens for each of B windows works on R = B*T rows, row
// r = b*T + t standing at absolute position position+t of window b.  The
// residual stream h is fp32 [R, d]; every operand a tensor-core product reads
// (the layer-normalised rows, the attention outputs, the GELU outputs) is the
// weights' 16-bit type, [R, Kp] with Kp = roundup(K, 32) and the pad columns
// zero.  Caches are the weights' 16-bit type.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace wsp {

enum class Storage : int { f16 = 1, bf16 = 2 };

inline int padded(int k) { return (k + 31) / 32 * 32; }

// ---------------------------------------------------------------- embed ---
struct EmbedArgs {
    const uint32_t* ring;   // [B][ring_stride] token slots
    int ring_stride;
    const int* position;    // device: tokens decoded before this step
    int tokens;             // T
    int rows;               // R
    int width;              // d
    int vocabulary;
    const void* token_table;        // 16-bit [V, token_stride]
    int token_stride;
    const float* position_table;    // fp32 [maxPositions, d]
    float* hidden;                  // fp32 [R, d]
    int* error;                     // bit 0: a token id outside the vocabulary
};
void launch_embed(Storage s, const EmbedArgs& a, cudaStream_t stream);

// ----------------------------------------------------------- layer norm ---
struct LayerNormArgs {
    const float* input;    // fp32 [*, d]; output row i reads input row i*row_step + row_offset
    int rows, width;
    int row_step, row_offset;
    const float* gamma;
    const float* beta;
    void* output;          // 16-bit [R, ld_output]
    int ld_output;
    float* hidden_copy;    // optional fp32 [R, d] copy of the normalised rows
};
void launch_layer_norm(Storage s, const LayerNormArgs& a, cudaStream_t stream);

// ------------------------------------------------------------- products ---
enum class Epilogue : int {
    qkv = 0,       // n<d: q (fp32) ; d<=n<2d: self key ; 2d<=n<3d: self value
    store = 1,     // fp32 out[r, n] = v
    residual = 2,  // fp32 out[r, n] += v
    gelu = 3,      // 16-bit out[r, n] = gelu(v)
    logits = 4,    // optional fp32 logits; masked argmax candidate per 16 columns
};

struct GemmArgs {
    const void* weight;   // 16-bit [N, Kp]
    const void* input;    // 16-bit [R, Kp]
    int n, rows, kp;
    const float* bias;    // [N] or null
    // store / residual / qkv(q part)
    float* out;
    int ld_out;
    // gelu
    void* out16;
    int ld_out16;
    // qkv
    int width;
    void* self_keys;      // this layer's [B][max_positions][d]
    void* self_values;
    int max_positions;
    int tokens;           // T
    const int* position;
    // logits
    float* logits;        // optional fp32 [R, ld_logits]
    int ld_logits;
    const float* mask;    // [N], nonzero = suppressed; null = none
    float* candidate_values;      // [R][n_tiles]
    uint32_t* candidate_indices;
};
int gemm_column_tiles(int n);
void launch_gemm(Storage s, Epilogue e, const GemmArgs& a, int sm_count, cudaStream_t stream);

// ------------------------------------------------------------ attention ---
struct AttentionArgs {
    const float* queries;    // fp32 [R, ld_queries]
    int ld_queries;
    const void* keys;        // 16-bit; key j of window b, head h at
    const void* values;      //   base + b*window_stride + j*key_stride + h*D
    long long key_stride;
    long long window_stride;
    int rows, tokens, heads, head_width;
    int causal;              // 1: row (b,t) sees keys 0..position+t
    const int* position;
    int key_count;           // non-causal: keys attended
    int chunk, splits;       // keys per CTA, CTAs per (row, head)
    float scale;
    float* partial;          // [R][H][S][D+2]: max, sum, unnormalised row
};
void launch_attention_partial(Storage s, const AttentionArgs& a, cudaStream_t stream);

struct CombineArgs {
    const float* partial;
    int rows, heads, head_width, splits;
    const float* bias;       // optional [d], added after normalising (cross V bias)
    void* output;            // 16-bit [R, ld_output]
    int ld_output;
};
void launch_attention_combine(Storage s, const CombineArgs& a, cudaStream_t stream);

// ---------------------------------------------------------------- argmax ---
struct ArgmaxFinalArgs {
    const float* candidate_values;
    const uint32_t* candidate_indices;
    int candidates;          // per row
    int rows;                // rows scanned
    int rows_per_window;     // window b owns rows b*rows_per_window ..; its last one is sampled
    int step_tokens;         // T: the sampled id lands in slot position + T
    uint32_t* row_tokens;    // optional [rows]
    uint32_t* ring;          // optional: ring[b*ring_stride + position + T]
    int ring_stride;
    const int* position;
};
void launch_argmax_final(const ArgmaxFinalArgs& a, cudaStream_t stream);

// Standalone masked argmax over [rows, length] fp32 logits (Argmax.h:207-262).
void launch_argmax_rows(const float* logits, const float* mask, uint32_t* out, int rows,
                        int length, float* candidate_values, uint32_t* candidate_indices,
                        int groups_per_row, cudaStream_t stream);
int argmax_groups_per_row(int length);

// ------------------------------------------------------------- plumbing ---
void launch_advance_position(int* position, int tokens, cudaStream_t stream);
void launch_to_storage(Storage s, const float* in, void* out, long long count, cudaStream_t stream);

}  // namespace wsp
