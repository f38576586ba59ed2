// The decoder step as a list of fused ops, run by one persistent kernel.
//
// A step of T tokens for each of B windows works on R = B*T rows; row
// r = b*T + t stands at absolute position position+t of window b.  The host
// lowers recordDecoderStep (Lib/WhisperEACP/Decoder/Decoder.cpp:151-177) and
// decoderLayer (:73-115) into StepOps:
//
//   embed                       h = token_table[id] + position_table[p]
//   (norm)                      with more than a few rows, each LayerNorm
//                               below runs once as its own op into 16-bit
//                               rows instead of in every CTA's product
//   per layer
//     product  LN1 -> q,k,v     (k, v appended to the self cache)
//     self attention            causal over keys 0..position+t
//     product  out_proj + h     (residual)
//     product  LN2 -> cross q
//     cross attention           the encoder rows' keys and values streamed
//                               through the ring, split over warps; the
//                               splits of a (row, head) joined by the last
//                               to finish
//     product  out_proj + h
//     product  LN3 -> fc1, GELU
//     product  fc2 + h
//   logits                      LN, h . token_table^T, masked argmax candidates;
//                               the last CTA to finish folds them, writes the
//                               sampled ids and advances the position
//
// with a grid-wide barrier after each op.  The decode kernel runs the list
// once per step for as many steps as it is given, so a whole greedy decode is
// one launch.

#pragma once

#include "common.cuh"

namespace wsp {

// Consumer warps of a decode-kernel CTA (a producer warp streams weights).
constexpr int kStepWarps = 7;
// Most keys one cross-attention stream unit carries, and most splits of a
// (row, head).
constexpr int kMaxCrossUnitKeys = 256;
constexpr int kMaxCrossSplits = 32;
// Keys of the score row of a self-attention warp (>= max_positions).
constexpr int kSelfWarpKeys = 512;
// Splits of a deferred q/k/v join a warp loads before summing.
constexpr int kDeferLoads = 8;
// Join counters per op of a split tensor-core product.
constexpr int kSplitSlots = 128;
// Most stages of a CTA's weight-stream ring (as many as shared memory holds).
constexpr int kMaxStreamStages = 12;

enum OpKind : int {
    kOpEmbed = 0,
    kOpProduct = 1,
    kOpSelfAttention = 2,
    kOpCrossAttention = 3,
    kOpLogits = 4,
    kOpNone = 5,
    kOpNorm = 6,
};
enum EpilogueKind : int { kEpQkv = 0, kEpStore = 1, kEpResidual = 2, kEpGelu = 3, kEpPartial = 4 };

// state words (int): position, error bits, abort, steps done, all windows
// ended, and where the first bounded wait gave up: its kind (WaitKind), CTA,
// and op or unit index
enum StateWord : int {
    kPosition = 0, kError = 1, kAbort = 2, kStepsDone = 3, kAllEnded = 4,
    kFailKind = 5, kFailCta = 6, kFailWhere = 7, kStateWords = 8
};
enum WaitKind : int { kWaitGrid = 1, kWaitUnit = 2, kWaitEmpty = 3, kWaitDrain = 4, kWaitArmed = 5, kWaitJoin = 6 };
enum ErrorBit : int { kErrToken = 1, kErrBarrierTimeout = 2 };

// Weight matrices are stored fragment-packed: the 16-row tiles of an [n, kp]
// matrix one after another, each as kp/32 chunks of 1 KB.  In a chunk, lane
// l = 4*(row%8) + (k%32)/8 of an m16n8k16 A fragment owns two 16-byte
// pieces -- eight k of row row%8 at byte 16 l, eight k of row row%8 + 8 at
// 512 + 16 l -- so each of a warp's two 16-byte loads of a chunk reads 512
// contiguous bytes, free of bank conflicts.  A tile is one contiguous block a
// bulk copy moves whole.
__host__ __device__ inline size_t packed_offset(int n, int k, int chunks) {
    const int tile = n >> 4, row = n & 15, chunk = k >> 5, kk = k & 31;
    const int lane = (row & 7) * 4 + (kk >> 3);
    return (((size_t)tile * chunks + chunk) * 2 + (row >> 3)) * 256 + lane * 8 + (kk & 7);
}

// With many rows (the tensor-core products), weights and 16-bit activations
// are laid out for tcgen05: K-major blocks of 64 columns (128 bytes a row)
// in 8-row atoms whose 16-byte pieces rotate by row % 8 (the 128-byte
// swizzle).  A weight matrix is 128-row tiles of kp/64 such blocks (16 KB
// each); an activation matrix is kp/64 blocks of act_rows rows.
__host__ __device__ inline size_t umma_offset(int n, int k, int kblocks) {
    const int tile = n >> 7, r = n & 127, kb = k >> 6, c = (k >> 3) & 7;
    return (((size_t)tile * kblocks + kb) * 128 + r) * 64 + ((c ^ (r & 7)) << 3) + (k & 7);
}
__host__ __device__ inline size_t act_offset(int r, int c, int act_rows) {
    return ((size_t)(c >> 6) * act_rows + r) * 64 + ((((c >> 3) & 7) ^ (r & 7)) << 3) + (c & 7);
}

struct StepOp {
    int kind;
    int epilogue;
    // products
    const void* weight;     // 16-bit fragment-packed [n, kp]
    int n, kp;
    const float* bias;      // [n] or null
    const float* gamma;     // non-null: the input is LayerNorm(h) with this gain ...
    const float* beta;      // ... and offset
    const void* input16;    // gamma == null: 16-bit input rows [R, ld_input]
    int ld_input;
    void* out;              // fp32 [R, ld_out] (q, residual) or 16-bit (gelu)
    int ld_out;
    void* self_keys;        // qkv: this layer's caches [B][max_positions][d]
    void* self_values;
    // attention
    const void* keys;       // 16-bit.  self: key j of window b, head h at
    const void* values;     //   base + b*window_stride + j*key_stride + h*D.
                            // cross: keys = this layer's block; key j of
                            // window b, head h is the row at base +
                            // b*window_stride + h*head_stride + j*key_stride,
                            // its D key values then its D value values
    long long key_stride;
    long long window_stride;
    long long head_stride;
    int key_count;          // cross: encoder rows attended
    int chunk;              // cross: keys per stream unit (<= kMaxCrossUnitKeys)
    int span;               // cross: units per split
    int splits;             // cross: splits per (row, head) (<= kMaxCrossSplits)
    const float* value_bias;  // cross: v_proj bias, added after normalising
    int slice;              // kEpStore: rows of a head (D), each head padded to a whole tile
    // norm: LayerNorm(gamma, beta) of norm_rows rows of h -- row i reads h
    // row i*norm_step + norm_offset -- into 16-bit rows `out` [norm_rows,
    // ld_out] (zero past the width), and into fp32 norm_hidden when given.
    // A product or the logits with input16 set and no gamma read such rows.
    int norm_rows, norm_step, norm_offset;
    float* norm_hidden;
    int norm_umma;          // norm: write the tensor-core activation layout
    // Attention ops with out_weight set (a few rows, 64-wide heads): each
    // (row, head) also applies its head's 64 columns of the attention
    // out-projection (fragment-packed [d, kpd], bias left out) to the head's
    // attended values and writes the d results to out_partial [H][R][d]; the
    // op after it adds them, so the out-projection is no op of its own.
    const void* out_weight;
    float* out_partial;
    // LayerNorm prologues and norm ops: the rows normalised are norm_input
    // (p.h when null) plus, with addend_count > 0, addend_bias and addends +
    // j * addend_stride (row-major [R][d]) for j = 0 .. addend_count-1 in
    // that order; the CTA that holds a row tile's first weight tile (a norm
    // op: the row's CTA) writes those sums, the new residual rows, to
    // sum_out.  With addend_tile_rows > 0 the addends are a tensor-core
    // product's split partials instead ([split][weight tile][row][128],
    // addend_tile_rows rows a tile), summed in split order and then added
    // with the bias: the product's own join, moved into the norm after it.
    const float* norm_input;
    const float* addends;
    int addend_count;
    long long addend_stride;
    const float* addend_bias;
    float* sum_out;
    // q/k/v products (a few rows): prefetch into L2 the self keys and values
    // the self attention after it reads.
    int prefetch_keys;
    int addend_tile_rows;
    // Tensor-core products: K splits of each tile's inner size.  With more
    // than one (only when all the items fit one wave of CTAs), each item
    // writes fp32 partials to p.partial_d [split][n_pad][rows_pad], the
    // tile's splits meet, and each sums its share of the rows in split order
    // and applies the epilogue.
    int ksplit;
    // A split product whose join is left to the op after it: a q/k/v
    // product's to the self attention (single-token steps of the tensor-core
    // path), a residual product's to the norm op (addend_tile_rows above).
    // The product stops at its partials.  The self attention sums the
    // partials of its (row, head)
    // -- qkv_splits of them, qkv_split_stride floats apart, rows
    // qkv_row_stride apart in a weight tile's block, in split order, then
    // qkv_bias -- appends k and v to the caches and attends with q.
    int defer_join;
    // A few-row product split over its inner size (mma.sync form): kparts
    // items a tile, each over kp / kparts of K, writing its sums without the
    // bias (kEpPartial) to out [part][R][ld_out]; the LayerNorm prologue of
    // the op that reads them adds the parts in order (its addends).
    int kparts;
    const float* qkv_partial;
    long long qkv_split_stride;
    int qkv_row_stride;
    int qkv_splits;
    const float* qkv_bias;
};

struct StepParams {
    int windows, tokens, rows;          // B, T, R
    int width, heads, head_width, ffn, vocabulary, kpd;
    int max_positions, ring_stride;
    // Tensor-core products: weights and activations in the umma layouts
    // above; act_rows rows an activation block; a product item covers
    // umma_rows rows (<= 256) of 128 weight rows.
    int umma, act_rows, umma_rows;
    // Input rows of a general product's or the logits' tile: 8 * tile_columns
    // (1, 2 or 4; 0: chosen from the rows).
    int tile_columns;
    float* partial_d;                   // fp32 split-K partials of a tensor-core product
    unsigned* split_counters;           // [n_ops][kSplitSlots] split arrivals (zero at launch)
    int umma_x_stages, umma_x_stage_bytes;  // the activation ring in the work area
    int umma_blocks;                    // 16 KB weight k-blocks a stream unit carries
    float scale;                        // 1/sqrt(D), on the scores (DecoderShape.cpp:19-26)
    int out_rows, row_step, row_offset; // logits rows: row i reads h row i*row_step + row_offset

    uint32_t* ring;                     // [B][ring_stride] token slots
    int* state;                         // StateWord
    const void* token_table;            // 16-bit fragment-packed [V, kpd]
    const float* position_table;        // fp32 [max_positions, d]
    const float* final_gamma;
    const float* final_beta;
    float* h;                           // fp32 [R, d] residual stream
    float* q;                           // fp32 [R, d]
    void* attn16;                       // 16-bit [R, kpd]
    void* ffn16;                        // 16-bit [R, kpf]
    float* partial;                     // cross partials [R][H][S][D+2]
    unsigned* combine_counters;         // [R*H]
    unsigned* logits_counter;           // [1]
    float* candidate_values;            // [out_rows][gridDim]
    uint32_t* candidate_indices;
    unsigned* barrier;                  // [0] arrivals since the launch began
    unsigned long long* profile;        // optional [n_ops+1] globaltimer stamps of step 0
    const float* mask;                  // logits mask (nonzero = suppressed) or null
    float* logits_out;                  // optional fp32 [out_rows, V]
    float* hidden_out;                  // optional fp32 [out_rows, d]
    uint32_t* row_tokens;               // optional [out_rows] greedy ids
    uint8_t* ended;                     // [B] window produced the stop token
    int write_ring;
    int steps;
    uint32_t stop_token;
    int stop_enabled;
    const StepOp* ops;
    int n_ops;
    int stage_bytes;                    // bytes of a weight-stream stage (multiple of 1 KB)
    int stages;                         // stages in the ring
    // The weight units each CTA streams in one step, in order: CTA c's are
    // schedule[schedule_offsets[c] .. schedule_offsets[c+1]).
    const struct ScheduleEntry* schedule;
    const unsigned* schedule_offsets;
};

// Item (m tile of 128 weight rows, row group, K split) of a tensor-core
// product: CTA c takes items c, c + grid, ...; split `split` covers k-blocks
// [kb0, kb1) of the kp/64.
struct UmmaItem {
    int m, r0, rows, split, kb0, kb1;
};
__host__ __device__ inline UmmaItem umma_item(const StepParams& p, const StepOp& op, int item) {
    const int m_tiles = (op.n + 127) / 128, groups = (p.rows + p.umma_rows - 1) / p.umma_rows;
    const int kblocks = op.kp / 64, ks = op.ksplit > 1 ? op.ksplit : 1, per = (kblocks + ks - 1) / ks;
    UmmaItem u;
    u.m = item % m_tiles;
    const int rest = item / m_tiles;
    u.r0 = (rest % groups) * p.umma_rows;
    u.rows = p.rows - u.r0 < p.umma_rows ? p.rows - u.r0 : p.umma_rows;
    u.split = rest / groups;
    u.kb0 = u.split * per;
    u.kb1 = u.kb0 + per < kblocks ? u.kb0 + per : kblocks;
    return u;
}

// One weight-stream unit: a 16-byte aligned source and its size in bytes.
// Units hold what no op of the launch writes (weights, the token table, the
// cross keys and values), so the producer may fetch them any time ahead.
// An entry with kPrefetchOnly set in `bytes` is no unit: the producer asks
// L2 for that range (an op's parameters and the like) and moves on.
struct __align__(16) ScheduleEntry {
    unsigned long long source;
    unsigned long long bytes;
};
constexpr unsigned long long kPrefetchOnly = 1ull << 32;

__host__ __device__ inline ScheduleEntry schedule_entry(const void* src, unsigned bytes) {
    return ScheduleEntry{(unsigned long long)(size_t)src, (unsigned long long)bytes};
}

}  // namespace wsp
