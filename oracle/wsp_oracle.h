/*
 * wsp_oracle.h -- CPU oracle for the Whisper decoder token loop.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the checker: tests/, the
 * smoke() entry of __graft_entry__.py and bench.py's cpu_baseline leg (and
 * its --impl reference arm) may load it.  The product path (the CUDA library
 * under whispereacp_b200/) never links, loads or calls it.
 *
 * It restates, in double precision, the scalar reference decoder that
 * WhisperEACP's own test suite asserts its GPU decoder against:
 *
 *   Tests/Decoder/Common.h:258-325   referenceDecoderAttention
 *   Tests/Decoder/Common.h:360-468   referenceDecode
 *   Tests/Decoder/Common.h:473-488   syntheticEncoderOutput
 *   Tests/Decoder/Common.h:490-500   argmaxRow
 *   Tests/Encoder/Common.h:390-393   referenceGelu
 *   Tests/Encoder/Common.h:444-479   referenceLayerNorm
 *   Tests/Encoder/Common.h:483-507   referenceLinear
 *   Tests/Encoder/Common.h:148-156   shiftedValues
 *   Tests/Kernels/Common.h:79-88     spreadValues
 *   Tests/Kernels/ArgmaxTests.cpp:20-35  argmaxReference (masked)
 *   Lib/WhisperEACP/Core/Utils/Half.cpp:8-78  packHalf / halfToFloat
 *
 * Two forms of the forward pass are provided.  wspo_reference_decode runs a
 * whole token sequence from position 0 exactly as referenceDecode does.  The
 * session form keeps the keys and values in double and appends a step at a
 * time; it performs the same per-element arithmetic in the same order, so
 * its rows are bit-identical to the full form's (a test asserts this), and it
 * makes hundreds of steps over 1500 encoder rows affordable.
 *
 * Parity pin: oracle/Makefile compiles the reference's own scalar decoder
 * from the lines where they lie in the reference checkout into
 * oracle/_ref/libref_decoder.so, and tests/golden/make_golden.py uses it to
 * write the fixtures this oracle is checked against.
 */
#ifndef WSP_ORACLE_H
#define WSP_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* DecoderShape (Lib/WhisperEACP/Decoder/DecoderShape.h:20-83). */
typedef struct wspo_shape {
    int width;
    int heads;
    int layers;
    int feed_forward_width;
    int vocabulary_size;
    int max_positions;
    int cross_positions;
} wspo_shape;

/*
 * The model is a flat array of float pointers in this order (the order of
 * DecoderWeights / DecoderLayerWeights, DecoderWeights.h:25-160):
 *
 *   [0] embed_tokens [V,d]   [1] embed_positions [maxPositions,d]
 *   [2] layer_norm.weight    [3] layer_norm.bias
 *   then per layer l, 24 pointers starting at 4 + 24*l:
 *     self:  norm.w norm.b q.w q.b k.w v.w v.b out.w out.b        (0..8)
 *     cross: norm.w norm.b q.w q.b k.w v.w v.b out.w out.b        (9..17)
 *     final_layer_norm.w final_layer_norm.b fc1.w fc1.b fc2.w fc2.b (18..23)
 */
enum {
    WSPO_TOKEN_EMBEDDING = 0,
    WSPO_POSITIONAL_EMBEDDING = 1,
    WSPO_FINAL_NORM_WEIGHT = 2,
    WSPO_FINAL_NORM_BIAS = 3,
    WSPO_GLOBAL_TENSORS = 4,
    WSPO_LAYER_TENSORS = 24
};

int wspo_tensor_count(const wspo_shape* shape);

/*
 * Full-sequence reference: tokens[0..count) at positions 0..count-1.
 * encoder is [cross_rows, width] float (the shape's cross_positions is
 * ignored in favour of cross_rows, as a reduced-context shape would be).
 * hidden receives [count, width], logits [count, vocabulary] (either may be
 * NULL).  threads <= 1 runs serially; the result does not depend on it.
 */
int wspo_reference_decode(const wspo_shape* shape, const float* const* tensors,
                          const float* encoder, int cross_rows,
                          const int32_t* tokens, int count,
                          double* hidden, double* logits, int threads);

/* Incremental (KV-cached) form. */
typedef struct wspo_session wspo_session;

wspo_session* wspo_session_new(const wspo_shape* shape,
                               const float* const* tensors, int threads);
void wspo_session_free(wspo_session* session);
/* Projects the cross keys/values from cross_rows encoder rows; position -> 0. */
int wspo_session_begin(wspo_session* session, const float* encoder,
                       int cross_rows);
/* Appends count tokens; returns -1 (and changes nothing) past max_positions. */
int wspo_session_step(wspo_session* session, const int32_t* tokens, int count,
                      double* hidden, double* logits);
int wspo_session_position(const wspo_session* session);

/*
 * Masked argmax, ArgmaxTests.cpp:20-35: the first index holding the largest
 * logit among mask[j] == 0; a row with nothing allowed gives 0.  mask may be
 * NULL (nothing suppressed), which is argmaxRow (Common.h:490-500).
 */
void wspo_masked_argmax_f64(const double* logits, const float* mask,
                            int rows, int row_length, uint32_t* out);
void wspo_masked_argmax_f32(const float* logits, const float* mask,
                            int rows, int row_length, uint32_t* out);

/* Generators of the reference's test fixtures. */
void wspo_spread_values(float* out, int count, uint32_t seed, float range);
void wspo_shifted_values(float* out, int count, uint32_t seed, float range);
void wspo_synthetic_encoder_output(float* out, int positions, int width);

/* Number formats. */
uint16_t wspo_pack_half(float value);
float wspo_half_to_float(uint16_t bits);
uint16_t wspo_pack_bfloat16(float value);
float wspo_bfloat16_to_float(uint16_t bits);

#ifdef __cplusplus
}
#endif

#endif
