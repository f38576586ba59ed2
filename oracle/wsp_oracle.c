/*
 * wsp_oracle.c -- double-precision CPU oracle for the decoder token loop.
 *
 * TEST INFRASTRUCTURE ONLY (see wsp_oracle.h): never part of the product.
 *
 * Every function names the reference lines it restates.  The arithmetic is
 * kept in the reference's order -- each sum starts where the reference's
 * starts and walks its terms in the same direction -- so that this oracle
 * and the reference's own scalar decoder, compiled from its sources by
 * oracle/Makefile, agree to the last bit (tests/test_oracle_golden.py).
 */
#include "wsp_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

/* ------------------------------------------------------------------------ */
/* Mersenne twister, the 32-bit MT19937 of Matsumoto and Nishimura (1998),    */
/* which is what std::mt19937 is specified to be.                            */
/* ------------------------------------------------------------------------ */

typedef struct {
    uint32_t state[624];
    int next;
} mt19937;

static void mt_seed(mt19937* engine, uint32_t seed)
{
    engine->state[0] = seed;
    for (int i = 1; i < 624; ++i) {
        uint32_t previous = engine->state[i - 1];
        engine->state[i] = 1812433253u * (previous ^ (previous >> 30)) + (uint32_t)i;
    }
    engine->next = 624;
}

static uint32_t mt_next(mt19937* engine)
{
    if (engine->next >= 624) {
        for (int i = 0; i < 624; ++i) {
            uint32_t y = (engine->state[i] & 0x80000000u) |
                         (engine->state[(i + 1) % 624] & 0x7fffffffu);
            uint32_t twisted = y >> 1;
            if (y & 1u)
                twisted ^= 0x9908b0dfu;
            engine->state[i] = engine->state[(i + 397) % 624] ^ twisted;
        }
        engine->next = 0;
    }
    uint32_t y = engine->state[engine->next++];
    y ^= y >> 11;
    y ^= (y << 7) & 0x9d2c5680u;
    y ^= (y << 15) & 0xefc60000u;
    y ^= y >> 18;
    return y;
}

/* Tests/Kernels/Common.h:79-88 -- range * ((float)(e() % 2001) / 1000 - 1). */
void wspo_spread_values(float* out, int count, uint32_t seed, float range)
{
    mt19937 engine;
    mt_seed(&engine, seed);
    for (int i = 0; i < count; ++i) {
        float unit = (float)(mt_next(&engine) % 2001u) / 1000.f - 1.f;
        out[i] = range * unit;
    }
}

/* Tests/Encoder/Common.h:148-156 -- spreadValues plus one (layer-norm gains). */
void wspo_shifted_values(float* out, int count, uint32_t seed, float range)
{
    wspo_spread_values(out, count, seed, range);
    for (int i = 0; i < count; ++i)
        out[i] += 1.f;
}

/* Tests/Decoder/Common.h:473-488. */
void wspo_synthetic_encoder_output(float* out, int positions, int width)
{
    for (int position = 0; position < positions; ++position)
        for (int column = 0; column < width; ++column) {
            double phase = 0.13 * position + 0.041 * column;
            out[position * width + column] =
                (float)(sin(phase) + 0.5 * cos(2.7 * phase));
        }
}

/* ------------------------------------------------------------------------ */
/* Number formats.                                                           */
/* ------------------------------------------------------------------------ */

static uint32_t float_bits(float value)
{
    uint32_t bits;
    memcpy(&bits, &value, sizeof bits);
    return bits;
}

static float bits_float(uint32_t bits)
{
    float value;
    memcpy(&value, &bits, sizeof value);
    return value;
}

/*
 * IEEE binary32 -> binary16, round to nearest even, overflow to infinity,
 * NaN kept quiet (Lib/WhisperEACP/Core/Utils/Half.cpp:8-56 states the same
 * rule).  Written from the format definition: the value is taken as an
 * integer significand and shifted right with a round-half-even on the bits
 * shifted out.
 */
uint16_t wspo_pack_half(float value)
{
    uint32_t bits = float_bits(value);
    uint16_t sign = (uint16_t)((bits >> 16) & 0x8000u);
    uint32_t magnitude = bits & 0x7fffffffu;

    if (magnitude >= 0x7f800000u) /* inf or NaN */
        return (uint16_t)(sign | 0x7c00u | (magnitude > 0x7f800000u ? 0x200u : 0u));

    if (magnitude < 0x00800000u) /* float zero or subnormal: below half's range */
        return sign;
    int exponent = (int)(magnitude >> 23) - 127; /* unbiased */
    if (exponent > 15)
        return (uint16_t)(sign | 0x7c00u);

    /*
     * value = significand * 2^(exponent - 23), significand a 24-bit integer.
     * A half normal keeps 10 fraction bits beside its exponent field (the
     * exponent and fraction are added so that a rounding carry moves the
     * exponent); a half subnormal counts units of 2^-24.
     */
    uint32_t significand;
    uint32_t base;
    int shift;
    if (exponent >= -14) {
        significand = magnitude & 0x7fffffu;
        base = (uint32_t)(exponent + 15) << 10;
        shift = 13;
    } else {
        significand = (magnitude & 0x7fffffu) | 0x800000u;
        base = 0;
        shift = -exponent - 1;
        if (shift > 24)
            return sign;
    }
    uint32_t kept = significand >> shift;
    uint32_t dropped = significand & ((1u << shift) - 1u);
    uint32_t half = 1u << (shift - 1);
    uint32_t result = base + kept;
    if (dropped > half || (dropped == half && (result & 1u)))
        result += 1u; /* may carry into the exponent, or up to infinity */
    if (result >= 0x7c00u)
        result = 0x7c00u;
    return (uint16_t)(sign | result);
}

float wspo_half_to_float(uint16_t bits)
{
    uint32_t sign = (uint32_t)(bits & 0x8000u) << 16;
    uint32_t exponent = (bits >> 10) & 0x1fu;
    uint32_t fraction = bits & 0x3ffu;
    if (exponent == 0x1fu)
        return bits_float(sign | 0x7f800000u | (fraction << 13));
    if (exponent == 0) {
        float magnitude = (float)fraction * (1.0f / 16777216.0f);
        return sign ? -magnitude : magnitude;
    }
    return bits_float(sign | ((exponent + 112u) << 23) | (fraction << 13));
}

/* binary32 -> bfloat16 (the top half), round to nearest even. */
uint16_t wspo_pack_bfloat16(float value)
{
    uint32_t bits = float_bits(value);
    if ((bits & 0x7fffffffu) > 0x7f800000u)
        return (uint16_t)((bits >> 16) | 0x40u);
    uint32_t rounding = 0x7fffu + ((bits >> 16) & 1u);
    return (uint16_t)((bits + rounding) >> 16);
}

float wspo_bfloat16_to_float(uint16_t bits)
{
    return bits_float((uint32_t)bits << 16);
}

/* ------------------------------------------------------------------------ */
/* The reference's building blocks.                                         */
/* ------------------------------------------------------------------------ */

#define LAYER_NORM_EPSILON 1e-5f /* LayerNorm::whisperEpsilon, LayerNorm.h:21 */

/* Tests/Encoder/Common.h:444-479: two-pass, centred variance. */
static void layer_norm(const double* rows, int row_count, int width,
                       const float* weight, const float* bias, double* out)
{
    for (int row = 0; row < row_count; ++row) {
        const double* x = rows + (size_t)row * width;
        double* y = out + (size_t)row * width;
        double mean = 0.0;
        for (int c = 0; c < width; ++c)
            mean += x[c];
        mean /= width;
        double variance = 0.0;
        for (int c = 0; c < width; ++c) {
            double centred = x[c] - mean;
            variance += centred * centred;
        }
        double scale = 1.0 / sqrt(variance / width + (double)LAYER_NORM_EPSILON);
        for (int c = 0; c < width; ++c)
            y[c] = (x[c] - mean) * scale * weight[c] + bias[c];
    }
}

/*
 * Tests/Encoder/Common.h:483-507: nn.Linear, weight [out, inner]; bias NULL for
 * k_proj.  Every output is its bias plus x[step] * w[step] added in step
 * order, exactly the reference's loop.  Only the order in which outputs are
 * visited differs: tiles of LINEAR_ROWS input rows x LINEAR_COLUMNS weight
 * rows, so a tile's weight rows stay in cache across its input rows, with
 * four outputs' sums carried side by side (each still in step order).  The
 * results are bit-identical to the one-output-at-a-time loop.
 */
#define LINEAR_ROWS 32
#define LINEAR_COLUMNS 16
/* One output: bias + x . w in step order. */
static double linear_one(const double* x, const float* w, const float* bias, int column, int inner)
{
    double total = bias == NULL ? 0.0 : (double)bias[column];
    for (int step = 0; step < inner; ++step)
        total += x[step] * (double)w[step];
    return total;
}

static void linear(const double* input, int row_count, int inner,
                   const float* weight, const float* bias, int out_width,
                   double* out, int threads)
{
    long total_outputs = (long)row_count * out_width;
    long row_tiles = (row_count + LINEAR_ROWS - 1) / LINEAR_ROWS;
    long column_tiles = (out_width + LINEAR_COLUMNS - 1) / LINEAR_COLUMNS;
    long tiles = row_tiles * column_tiles;
#pragma omp parallel for schedule(dynamic, 1) num_threads(threads > 0 ? threads : 1) if (threads > 1 && total_outputs > 4096)
    for (long tile = 0; tile < tiles; ++tile) {
        int c0 = (int)(tile % column_tiles) * LINEAR_COLUMNS;
        int r0 = (int)(tile / column_tiles) * LINEAR_ROWS;
        int c1 = c0 + LINEAR_COLUMNS < out_width ? c0 + LINEAR_COLUMNS : out_width;
        int r1 = r0 + LINEAR_ROWS < row_count ? r0 + LINEAR_ROWS : row_count;
        int row = r0;
        /* two input rows by four weight rows: eight sums, each in step order */
        for (; row + 2 <= r1; row += 2) {
            const double* x = input + (size_t)row * inner;
            const double* x2 = x + inner;
            double* y = out + (size_t)row * out_width;
            double* y2 = y + out_width;
            int column = c0;
            for (; column + 4 <= c1; column += 4) {
                const float* w0 = weight + (size_t)column * inner;
                const float* w1 = w0 + inner;
                const float* w2 = w1 + inner;
                const float* w3 = w2 + inner;
                double b0 = bias == NULL ? 0.0 : (double)bias[column];
                double b1 = bias == NULL ? 0.0 : (double)bias[column + 1];
                double b2 = bias == NULL ? 0.0 : (double)bias[column + 2];
                double b3 = bias == NULL ? 0.0 : (double)bias[column + 3];
                double t0 = b0, t1 = b1, t2 = b2, t3 = b3;
                double u0 = b0, u1 = b1, u2 = b2, u3 = b3;
                for (int step = 0; step < inner; ++step) {
                    double xv = x[step], xw = x2[step];
                    double v0 = w0[step], v1 = w1[step], v2 = w2[step], v3 = w3[step];
                    t0 += xv * v0;
                    t1 += xv * v1;
                    t2 += xv * v2;
                    t3 += xv * v3;
                    u0 += xw * v0;
                    u1 += xw * v1;
                    u2 += xw * v2;
                    u3 += xw * v3;
                }
                y[column] = t0; y[column + 1] = t1; y[column + 2] = t2; y[column + 3] = t3;
                y2[column] = u0; y2[column + 1] = u1; y2[column + 2] = u2; y2[column + 3] = u3;
            }
            for (; column < c1; ++column) {
                const float* w = weight + (size_t)column * inner;
                y[column] = linear_one(x, w, bias, column, inner);
                y2[column] = linear_one(x2, w, bias, column, inner);
            }
        }
        for (; row < r1; ++row) {
            const double* x = input + (size_t)row * inner;
            double* y = out + (size_t)row * out_width;
            int column = c0;
            for (; column + 4 <= c1; column += 4) {
                const float* w0 = weight + (size_t)column * inner;
                const float* w1 = w0 + inner;
                const float* w2 = w1 + inner;
                const float* w3 = w2 + inner;
                double t0 = bias == NULL ? 0.0 : (double)bias[column];
                double t1 = bias == NULL ? 0.0 : (double)bias[column + 1];
                double t2 = bias == NULL ? 0.0 : (double)bias[column + 2];
                double t3 = bias == NULL ? 0.0 : (double)bias[column + 3];
                for (int step = 0; step < inner; ++step) {
                    double xv = x[step];
                    t0 += xv * (double)w0[step];
                    t1 += xv * (double)w1[step];
                    t2 += xv * (double)w2[step];
                    t3 += xv * (double)w3[step];
                }
                y[column] = t0; y[column + 1] = t1; y[column + 2] = t2; y[column + 3] = t3;
            }
            for (; column < c1; ++column)
                y[column] = linear_one(x, weight + (size_t)column * inner, bias, column, inner);
        }
    }
}

/* Tests/Encoder/Common.h:390-393. */
static double gelu(double x)
{
    return 0.5 * x * (1.0 + erf(x / sqrt(2.0)));
}

/*
 * Tests/Decoder/Common.h:258-325, with the queries' absolute positions made
 * explicit: query i stands at first_position + i, and when causal it sees
 * keys 0..first_position+i.  The full-sequence form passes first_position 0,
 * which is the reference's `visible = query + 1`.
 */
static void attention(const double* queries, int query_count,
                      const double* keys, const double* values, int key_count,
                      int first_position, int causal, int width, int heads,
                      double* output, int threads)
{
    int head_width = width / heads;
    double scale = 1.0 / sqrt((double)head_width);
    int pairs = heads * query_count;

#pragma omp parallel num_threads(threads > 0 ? threads : 1) if (threads > 1 && pairs > 1)
    {
        double* row = (double*)malloc(sizeof(double) * (size_t)(key_count > 0 ? key_count : 1));
#pragma omp for schedule(static)
        for (int pair = 0; pair < pairs; ++pair) {
            int head = pair / query_count;
            int query = pair % query_count;
            int head_column = head * head_width;
            int visible = causal ? first_position + query + 1 : key_count;
            double largest = -INFINITY;

            for (int key = 0; key < visible; ++key) {
                double total = 0.0;
                for (int channel = 0; channel < head_width; ++channel)
                    total += queries[(size_t)query * width + head_column + channel] *
                             keys[(size_t)key * width + head_column + channel];
                row[key] = scale * total;
                largest = largest < row[key] ? row[key] : largest;
            }
            double total = 0.0;
            for (int key = 0; key < visible; ++key) {
                row[key] = exp(row[key] - largest);
                total += row[key];
            }
            for (int channel = 0; channel < head_width; ++channel) {
                double weighted = 0.0;
                for (int key = 0; key < visible; ++key)
                    weighted += row[key] * values[(size_t)key * width + head_column + channel];
                output[(size_t)query * width + head_column + channel] = weighted / total;
            }
        }
        free(row);
    }
}

int wspo_tensor_count(const wspo_shape* shape)
{
    return WSPO_GLOBAL_TENSORS + WSPO_LAYER_TENSORS * shape->layers;
}

#define LAYER(tensors, l, i) ((tensors)[WSPO_GLOBAL_TENSORS + WSPO_LAYER_TENSORS * (l) + (i)])

/* ------------------------------------------------------------------------ */
/* Session: the KV-cached form.                                              */
/* ------------------------------------------------------------------------ */

struct wspo_session {
    wspo_shape shape;
    const float* const* tensors;
    int threads;
    int position;
    int cross_rows;
    double* self_keys;    /* [layers][max_positions][width] */
    double* self_values;
    double* cross_keys;   /* [layers][cross_positions][width] */
    double* cross_values;
};

wspo_session* wspo_session_new(const wspo_shape* shape,
                               const float* const* tensors, int threads)
{
    wspo_session* s = (wspo_session*)calloc(1, sizeof *s);
    if (s == NULL)
        return NULL;
    s->shape = *shape;
    s->tensors = tensors;
    s->threads = threads;
    size_t self = (size_t)shape->layers * shape->max_positions * shape->width;
    size_t cross = (size_t)shape->layers * shape->cross_positions * shape->width;
    s->self_keys = (double*)calloc(self ? self : 1, sizeof(double));
    s->self_values = (double*)calloc(self ? self : 1, sizeof(double));
    s->cross_keys = (double*)calloc(cross ? cross : 1, sizeof(double));
    s->cross_values = (double*)calloc(cross ? cross : 1, sizeof(double));
    if (!s->self_keys || !s->self_values || !s->cross_keys || !s->cross_values) {
        wspo_session_free(s);
        return NULL;
    }
    return s;
}

void wspo_session_free(wspo_session* s)
{
    if (s == NULL)
        return;
    free(s->self_keys);
    free(s->self_values);
    free(s->cross_keys);
    free(s->cross_values);
    free(s);
}

int wspo_session_position(const wspo_session* s)
{
    return s->position;
}

/* Decoder.cpp:121-146 (recordSequenceStart): cross K = E Wk^T, V = E Wv^T + bv. */
int wspo_session_begin(wspo_session* s, const float* encoder, int cross_rows)
{
    const wspo_shape* shape = &s->shape;
    int width = shape->width;
    if (cross_rows <= 0 || cross_rows > shape->cross_positions)
        return -1;
    size_t elements = (size_t)cross_rows * width;
    double* rows = (double*)malloc(sizeof(double) * elements);
    if (rows == NULL)
        return -1;
    for (size_t i = 0; i < elements; ++i)
        rows[i] = encoder[i];
    for (int l = 0; l < shape->layers; ++l) {
        double* keys = s->cross_keys + (size_t)l * shape->cross_positions * width;
        double* values = s->cross_values + (size_t)l * shape->cross_positions * width;
        linear(rows, cross_rows, width, LAYER(s->tensors, l, 13), NULL, width, keys, s->threads);
        linear(rows, cross_rows, width, LAYER(s->tensors, l, 14), LAYER(s->tensors, l, 15),
               width, values, s->threads);
    }
    free(rows);
    s->cross_rows = cross_rows;
    s->position = 0;
    return 0;
}

/*
 * One decoder step of `count` tokens at positions position..position+count-1
 * (Decoder.cpp:151-177 recordDecoderStep, Decoder.cpp:73-115 decoderLayer),
 * with the arithmetic of referenceDecode (Common.h:360-468).
 */
int wspo_session_step(wspo_session* s, const int32_t* tokens, int count,
                      double* hidden_out, double* logits_out)
{
    const wspo_shape* shape = &s->shape;
    const float* const* t = s->tensors;
    int width = shape->width;
    int ffn = shape->feed_forward_width;
    int threads = s->threads;

    if (count <= 0 || s->position + count > shape->max_positions || s->cross_rows <= 0)
        return -1;
    for (int i = 0; i < count; ++i)
        if (tokens[i] < 0 || tokens[i] >= shape->vocabulary_size)
            return -1;

    size_t rows = (size_t)count * width;
    double* hidden = (double*)malloc(sizeof(double) * rows);
    double* normalised = (double*)malloc(sizeof(double) * rows);
    double* queries = (double*)malloc(sizeof(double) * rows);
    double* attended = (double*)malloc(sizeof(double) * rows);
    double* projected = (double*)malloc(sizeof(double) * rows);
    double* feed = (double*)malloc(sizeof(double) * (size_t)count * ffn);
    if (!hidden || !normalised || !queries || !attended || !projected || !feed) {
        free(hidden); free(normalised); free(queries); free(attended); free(projected); free(feed);
        return -1;
    }

    const float* token_table = t[WSPO_TOKEN_EMBEDDING];
    const float* position_table = t[WSPO_POSITIONAL_EMBEDDING];
    for (int i = 0; i < count; ++i)
        for (int c = 0; c < width; ++c)
            hidden[(size_t)i * width + c] =
                (double)token_table[(size_t)tokens[i] * width + c] +
                (double)position_table[(size_t)(s->position + i) * width + c];

    int keys_after = s->position + count;
    for (int l = 0; l < shape->layers; ++l) {
        double* self_k = s->self_keys + (size_t)l * shape->max_positions * width;
        double* self_v = s->self_values + (size_t)l * shape->max_positions * width;
        double* cross_k = s->cross_keys + (size_t)l * shape->cross_positions * width;
        double* cross_v = s->cross_values + (size_t)l * shape->cross_positions * width;

        /* self attention: q, and k/v appended at rows position.. (Decoder.cpp:29-48) */
        layer_norm(hidden, count, width, LAYER(t, l, 0), LAYER(t, l, 1), normalised);
        linear(normalised, count, width, LAYER(t, l, 2), LAYER(t, l, 3), width, queries, threads);
        linear(normalised, count, width, LAYER(t, l, 4), NULL, width,
               self_k + (size_t)s->position * width, threads);
        linear(normalised, count, width, LAYER(t, l, 5), LAYER(t, l, 6), width,
               self_v + (size_t)s->position * width, threads);
        attention(queries, count, self_k, self_v, keys_after, s->position, 1, width,
                  shape->heads, attended, threads);
        linear(attended, count, width, LAYER(t, l, 7), LAYER(t, l, 8), width, projected, threads);
        for (size_t i = 0; i < rows; ++i)
            hidden[i] += projected[i];

        /* cross attention over the projected encoder rows (Decoder.cpp:53-68) */
        layer_norm(hidden, count, width, LAYER(t, l, 9), LAYER(t, l, 10), normalised);
        linear(normalised, count, width, LAYER(t, l, 11), LAYER(t, l, 12), width, queries, threads);
        attention(queries, count, cross_k, cross_v, s->cross_rows, 0, 0, width,
                  shape->heads, attended, threads);
        linear(attended, count, width, LAYER(t, l, 16), LAYER(t, l, 17), width, projected, threads);
        for (size_t i = 0; i < rows; ++i)
            hidden[i] += projected[i];

        /* feed forward (Decoder.cpp:106-114) */
        layer_norm(hidden, count, width, LAYER(t, l, 18), LAYER(t, l, 19), normalised);
        linear(normalised, count, width, LAYER(t, l, 20), LAYER(t, l, 21), ffn, feed, threads);
        for (size_t i = 0; i < (size_t)count * ffn; ++i)
            feed[i] = gelu(feed[i]);
        linear(feed, count, ffn, LAYER(t, l, 22), LAYER(t, l, 23), width, projected, threads);
        for (size_t i = 0; i < rows; ++i)
            hidden[i] += projected[i];
    }

    /* final layer norm and the tied logits (Decoder.cpp:170-176) */
    layer_norm(hidden, count, width, t[WSPO_FINAL_NORM_WEIGHT], t[WSPO_FINAL_NORM_BIAS], normalised);
    if (hidden_out != NULL)
        memcpy(hidden_out, normalised, sizeof(double) * rows);
    if (logits_out != NULL)
        linear(normalised, count, width, token_table, NULL, shape->vocabulary_size, logits_out, threads);

    s->position += count;
    free(hidden); free(normalised); free(queries); free(attended); free(projected); free(feed);
    return 0;
}

/* ------------------------------------------------------------------------ */
/* Full-sequence form: Tests/Decoder/Common.h:360-468.                       */
/* ------------------------------------------------------------------------ */

int wspo_reference_decode(const wspo_shape* shape, const float* const* tensors,
                          const float* encoder, int cross_rows,
                          const int32_t* tokens, int count,
                          double* hidden, double* logits, int threads)
{
    if (count <= 0 || count > shape->max_positions || cross_rows <= 0)
        return -1;
    wspo_shape local = *shape;
    if (cross_rows > local.cross_positions)
        local.cross_positions = cross_rows;
    wspo_session* s = wspo_session_new(&local, tensors, threads);
    if (s == NULL)
        return -1;
    int status = wspo_session_begin(s, encoder, cross_rows);
    if (status == 0)
        status = wspo_session_step(s, tokens, count, hidden, logits);
    wspo_session_free(s);
    return status;
}

/* ------------------------------------------------------------------------ */
/* Masked argmax: Tests/Kernels/ArgmaxTests.cpp:20-35.                       */
/* ------------------------------------------------------------------------ */

void wspo_masked_argmax_f64(const double* logits, const float* mask,
                            int rows, int row_length, uint32_t* out)
{
    for (int row = 0; row < rows; ++row) {
        const double* base = logits + (size_t)row * row_length;
        int best = -1;
        for (int index = 0; index < row_length; ++index) {
            if (mask != NULL && mask[index] != 0.f)
                continue;
            if (best < 0 || base[index] > base[best])
                best = index;
        }
        out[row] = (uint32_t)(best < 0 ? 0 : best);
    }
}

void wspo_masked_argmax_f32(const float* logits, const float* mask,
                            int rows, int row_length, uint32_t* out)
{
    for (int row = 0; row < rows; ++row) {
        const float* base = logits + (size_t)row * row_length;
        int best = -1;
        for (int index = 0; index < row_length; ++index) {
            if (mask != NULL && mask[index] != 0.f)
                continue;
            if (best < 0 || base[index] > base[best])
                best = index;
        }
        out[row] = (uint32_t)(best < 0 ? 0 : best);
    }
}
