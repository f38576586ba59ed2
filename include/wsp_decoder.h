/*
 * wsp_decoder.h -- the C ABI of the B200 decoder token loop.
 *
 * This is the thin layer the C++ host code of a Whisper runtime reaches CUDA
 * through: plain pointers, sizes and int status codes, no C++ or torch types.
 * Each entry point names the WhisperEACP interface (path:line within that
 * project) whose role it takes over; INTEGRATION.md shows the binding a
 * maintainer adds on the reference side.
 *
 * Conventions
 *   - Every function returns a wsp_status.  A failure leaves the decoder as it
 *     was (validation happens on the host before anything is launched, as in
 *     Decoder.cpp:276-289) and its text is readable through wsp_last_error()
 *     on the calling thread.
 *   - Pointers to data (encoder rows, tokens, logits, masks) may be host or
 *     device pointers; unified addressing decides which, and host buffers are
 *     copied in/out inside the call.
 *   - A decoder is bound to one device and is not thread-safe.  Several GPUs
 *     are driven by several decoders, one host thread (or process) each.
 *   - "windows" is the batch: independent 30 s windows decoded in lockstep,
 *     each with its own self- and cross-attention caches.  WhisperEACP decodes
 *     one window at a time; windows == 1 is its behaviour.
 */
#ifndef WSP_DECODER_H
#define WSP_DECODER_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define WSP_ABI_VERSION 1

typedef enum wsp_status {
    WSP_OK = 0,
    WSP_MODEL_ERROR = 1,      /* WSP::ModelError: shapes, capacities, tensors  */
    WSP_LOGIC_ERROR = 2,      /* std::logic_error: misuse (e.g. step before begin) */
    WSP_INVALID_ARGUMENT = 3, /* std::invalid_argument (Argmax.cpp:54-58)     */
    WSP_CUDA_ERROR = 4,
    WSP_OUT_OF_MEMORY = 5
} wsp_status;

/* Element types of tensors handed in, and the decoder's 16-bit storage. */
typedef enum wsp_dtype {
    WSP_FLOAT32 = 0,
    WSP_FLOAT16 = 1,
    WSP_BFLOAT16 = 2
} wsp_dtype;

/* DecoderShape, Lib/WhisperEACP/Decoder/DecoderShape.h:20-31. */
typedef struct wsp_decoder_shape {
    int32_t width;
    int32_t heads;
    int32_t layers;
    int32_t feed_forward_width;
    int32_t vocabulary_size;
    int32_t max_positions;   /* max_target_positions: the self-attention capacity */
    int32_t cross_positions; /* encoder rows a sequence may attend to            */
} wsp_decoder_shape;

typedef struct wsp_decoder wsp_decoder;

/* Text of the last failure on this thread ("" when none). */
const char* wsp_last_error(void);

/* Library build and device queries. */
int wsp_abi_version(void);
int wsp_device_count(int* count);

/*
 * Decoder construction and Decoder::prepare
 * (Lib/WhisperEACP/Decoder/Decoder.h:49-66, Decoder.cpp:179-227): sizes every
 * cache and intermediate once, for `windows` windows, on `device`.  storage
 * is the 16-bit type weights, activations and caches are kept in
 * (WSP_FLOAT16 or WSP_BFLOAT16); products accumulate in fp32.
 */
int wsp_decoder_create(const wsp_decoder_shape* shape, int device, int windows,
                       wsp_dtype storage, wsp_decoder** out);

/*
 * The same with the form of the products chosen: WSP_PRODUCTS_MMA (mma.sync
 * tiles of 16 weight rows), WSP_PRODUCTS_TCGEN05 (tcgen05 tiles of 128
 * weight rows against every window's row, accumulated in tensor memory;
 * widths in 64-column blocks, 64-wide heads and 16+ windows, else
 * WSP_MODEL_ERROR), or WSP_PRODUCTS_AUTO (what wsp_decoder_create does: the
 * faster for the window count, as measured on B200).  No counterpart in the
 * reference.
 */
enum { WSP_PRODUCTS_AUTO = 0, WSP_PRODUCTS_MMA = 1, WSP_PRODUCTS_TCGEN05 = 2 };
int wsp_decoder_create_products(const wsp_decoder_shape* shape, int device, int windows,
                                wsp_dtype storage, int products, wsp_decoder** out);
void wsp_decoder_destroy(wsp_decoder* decoder);

/*
 * One tensor of a decoder checkpoint under its HuggingFace name, the role of
 * DecoderWeights / DecoderLayerWeights (Lib/WhisperEACP/Decoder/
 * DecoderWeights.h:25-160, DecoderWeights.cpp:74-178): "model.decoder.
 * layers.3.encoder_attn.q_proj.weight" and the rest.  The data (host memory)
 * is narrowed to the decoder's storage type and laid out for the kernels.  A
 * wrong rank or extent is WSP_MODEL_ERROR naming the tensor; a name outside
 * "model.decoder." is ignored (a full Whisper file carries the encoder too).
 */
int wsp_decoder_set_tensor(wsp_decoder* decoder, const char* name, wsp_dtype dtype,
                           const int64_t* extents, int rank, const void* data);

/*
 * How wsp_decoder_set_tensor narrows the projection matrices and the token
 * table to the storage type.  WSP_NARROW_ROUND (the default): round to
 * nearest even.  WSP_NARROW_EXACT: the ExactHalf rule of DecoderWeights
 * (Lib/WhisperEACP/Model/SafeTensors.h:146-159, Decoder/DecoderWeights.cpp:
 * 149-178) -- a tensor is narrowed only when every value survives unchanged;
 * where the reference then keeps that tensor in fp32, this decoder, whose
 * kernels read 16-bit weights only, refuses it with WSP_MODEL_ERROR naming
 * the tensor and the first value that would change (Whisper's checkpoints,
 * fp16 values in fp32 containers, narrow exactly to float16).  Set it before
 * the tensors.
 */
enum { WSP_NARROW_ROUND = 0, WSP_NARROW_EXACT = 1 };
int wsp_decoder_set_narrowing(wsp_decoder* decoder, int mode);

/*
 * Of the tensors set so far, how many were narrowed inexactly, and the
 * largest absolute change any value took.  No counterpart in the reference.
 */
int wsp_decoder_narrowing(const wsp_decoder* decoder, int* inexact_tensors, double* largest_change);

/* WSP_MODEL_ERROR naming the first decoder tensor not yet set, else WSP_OK. */
int wsp_decoder_check_weights(const wsp_decoder* decoder);

/*
 * Decoder::beginSequence (Decoder.h:67-73, Decoder.cpp:229-268;
 * recordSequenceStart Decoder.cpp:121-146): for every window, projects the
 * cross-attention keys and values of every layer out of its encoder rows and
 * resets the position to zero.  encoder_rows is fp32
 * [windows, shape.cross_positions, width]; cross_positions is how many of
 * each window's rows the sequence attends to (0 = all).
 */
int wsp_decoder_begin_sequence(wsp_decoder* decoder, const float* encoder_rows,
                               int cross_positions);

/*
 * Decoder::step (Decoder.h:75-98, Decoder.cpp:270-308; recordDecoderStep
 * Decoder.cpp:151-177): appends token_count tokens to every window.
 *   tokens  uint32 [windows, token_count]
 *   logits  fp32 [windows, token_count, vocabulary] or NULL
 *   hidden  fp32 [windows, token_count, width] (the rows after the final layer
 *           norm, Decoder.h:109-115) or NULL
 *   argmax  uint32 [windows, token_count]: the unmasked greedy token of each
 *           row (the DecoderRun harness's Argmax, Tests/Decoder/Common.h:
 *           618-660), or NULL
 * A step past max_positions is WSP_MODEL_ERROR before anything is launched.
 */
int wsp_decoder_step(wsp_decoder* decoder, const uint32_t* tokens, int token_count,
                     float* logits, float* hidden, uint32_t* argmax);

/* Decoder::position / Decoder::crossPositions (Decoder.h:100-107). */
int wsp_decoder_position(const wsp_decoder* decoder, int* position);
int wsp_decoder_cross_positions(const wsp_decoder* decoder, int* cross_positions);

/*
 * Greedy search configuration, the generation config Whisper::load builds
 * (Lib/WhisperEACP/Whisper/Whisper.cpp:148-254): the prompt
 * (buildPrompt, :207-225), the two suppression masks (buildSuppressionMasks,
 * :227-254; fp32 [vocabulary], nonzero = suppressed; the first applies to the
 * prompt step only), the token limit (maximumTokens, 448 - prompt) and the
 * end-of-text id that stops a window.  The call first waits for any
 * transcription still queued on the decoder's stream, which reads the
 * previous masks and prompt.
 */
typedef struct wsp_generation_config {
    const uint32_t* prompt;
    int32_t prompt_length;
    const float* first_step_mask;
    const float* later_step_mask;
    int32_t maximum_tokens;
    uint32_t end_of_text;
    int32_t stop_at_end_of_text; /* 0: run every step (benchmarks)          */
} wsp_generation_config;

int wsp_decoder_set_generation(wsp_decoder* decoder, const wsp_generation_config* config);

/*
 * Whisper::decodeTranscript (Whisper.cpp:1361-1449) with encodeStep and
 * encodeSampling (:1169-1213) for every window: begins the sequence over
 * encoder_rows, decodes the prompt in one step, then one token a step, each
 * sampled by masked argmax straight into the device token ring the next step
 * embeds.  The step limit is min(maximum_tokens, max_positions - prompt + 1)
 * (Whisper.cpp:1375-1377).  tokens receives uint32 [windows, step limit] (the
 * sampled ids, end-of-text excluded) and counts int32 [windows] (each
 * window's transcript length: up to its first end-of-text when stopping on
 * it).  The prompt is one launch of the persistent decode kernel and every
 * later step runs inside a second launch, which samples each window's id
 * into the token ring the next step embeds, with no host round trip.
 */
int wsp_decoder_transcribe(wsp_decoder* decoder, const float* encoder_rows,
                           int cross_positions, uint32_t* tokens, int32_t* counts);

/*
 * The same search split for timing: enqueue begins the sequence and queues
 * `steps` sampled steps on the decoder's stream without waiting (no early
 * stop); read waits and copies the transcript out as transcribe does.
 */
int wsp_decoder_enqueue_transcribe(wsp_decoder* decoder, const float* encoder_rows,
                                   int cross_positions, int steps);
int wsp_decoder_read_transcript(wsp_decoder* decoder, uint32_t* tokens, int32_t* counts);

/* The CUDA stream every launch of this decoder goes to (a cudaStream_t). */
void* wsp_decoder_stream(wsp_decoder* decoder);
int wsp_decoder_synchronize(wsp_decoder* decoder);

/*
 * Per-kernel timing for measurement: runs `steps` single-token greedy steps
 * launch by launch with CUDA events around each kernel, and writes the mean
 * milliseconds per launch of each kernel class into ms[WSP_KERNEL_CLASSES]
 * and the number of launches per step into launches[WSP_KERNEL_CLASSES].
 */
enum {
    WSP_KERNEL_EMBED = 0,
    WSP_KERNEL_LAYER_NORM = 1,
    WSP_KERNEL_PROJECTION = 2,
    WSP_KERNEL_SELF_ATTENTION = 3,
    WSP_KERNEL_CROSS_ATTENTION = 4,
    WSP_KERNEL_ATTENTION_COMBINE = 5,
    WSP_KERNEL_LOGITS_ARGMAX = 6,
    WSP_KERNEL_ARGMAX_FINAL = 7,
    WSP_KERNEL_OTHER = 8,
    WSP_KERNEL_CLASSES = 9
};
int wsp_decoder_time_kernels(wsp_decoder* decoder, int steps, float* ms, int* launches);

/*
 * Mean cost of one grid-wide barrier of the persistent decode kernel, in
 * microseconds: one launch running `count` empty ops.
 */
int wsp_decoder_time_barriers(wsp_decoder* decoder, int count, float* microseconds);

/*
 * Clock cycles per step that CTA 0 of the decode kernel spent in each section
 * (waiting for weights, products, grid barriers, reductions and epilogues,
 * layer norms and row staging, attention, the ops as a whole with barriers
 * excluded, a fused cross query, a cross split join, a fused out-projection,
 * a self-attention item, the logits, a one- or two-row layer norm's loads
 * and the rest of it, the logits' vocabulary tiles and their fold), averaged
 * over the last wsp_decoder_time_kernels run; `count` entries (16 are
 * defined).
 */
int wsp_decoder_trace_cycles(const wsp_decoder* decoder, double* cycles, int count);

/*
 * Microseconds of each op of the decode step's op list (its work and the
 * grid barrier after it, from CTA 0's clock) and the op's kind (0 embed,
 * 1 product, 2 self attention, 3 cross attention, 4 logits, 6 layer norm),
 * averaged over the last wsp_decoder_time_kernels run.  Fills up to
 * `capacity` entries of each array (either may be NULL) and sets *count to
 * the ops in the list.  Measurement only; no counterpart in the reference.
 */
int wsp_decoder_op_times(const wsp_decoder* decoder, float* microseconds, int* kinds, int capacity, int* count);

/*
 * Milliseconds of the last transcription's three phases, from CUDA events on
 * the decoder's stream: ms[0] the sequence start (encoder-row narrowing and
 * the cross K/V product), ms[1] the prompt step's launch, ms[2] the launch
 * that runs every later step (0 when there was none).  Waits for them.
 * Measurement only; no counterpart in the reference.
 */
int wsp_decoder_phase_ms(wsp_decoder* decoder, float* ms);

/* Kernel launches of this library per transcription (wsp_decoder_transcribe). */
int wsp_decoder_step_launches(const wsp_decoder* decoder, int* launches);

/*
 * Argmax::encode (Lib/WhisperEACP/Kernels/Argmax.h:207-262,
 * Argmax.cpp:47-80): indices[row] = the first j maximising
 * logits[row*row_length + j] over mask[j] == 0; a row with everything
 * suppressed gives 0.  logits, mask and indices are device pointers; stream
 * is a cudaStream_t (NULL: the legacy stream).  The call waits for its
 * result.
 */
int wsp_argmax(const float* logits, const float* mask, uint32_t* indices, int row_count,
               int row_length, void* stream);

/*
 * wsp_argmax for callers that must not allocate device memory: the same
 * masked argmax, the same result, but no cudaMalloc, cudaMallocAsync,
 * cudaFree or allocating library call.  No counterpart in the reference.
 * It is for host code that cannot enter the CUDA allocator -- a real-time
 * audio thread, where an allocation may block on driver locks or wait on
 * other work in the stream's pool, or a runtime that has already reserved
 * every byte of its memory budget.
 *
 * Its scratch is a fixed 512 KB array inside this library (static device
 * memory, loaded with the module), so row_count x ceil(row_length / 2048)
 * may be at most WSP_ARGMAX_NO_ALLOC_MAX_GROUPS (65536: e.g. 2520 rows of
 * 51866); more is WSP_INVALID_ARGUMENT before anything is launched.  Nothing
 * in the scratch has to start at zero.
 *
 * The first call on a device looks the scratch's address up
 * (cudaGetSymbolAddress) with that device current and remembers it: make
 * that first call during set-up, before any stream capture.  The address
 * lives as long as the device's context: after cudaDeviceReset (or anything
 * else that destroys the primary context) the remembered address is stale,
 * so do not call this entry point again in that process.  The call works
 * on the current device; logits, mask and indices are device pointers there.
 * It queues two kernels on `stream` (NULL: the legacy stream) and returns
 * without waiting; indices hold the result once the stream has passed them.
 *
 * Every call on a device shares the one scratch: two calls whose work
 * overlaps on the device (different streams, or different host threads,
 * without ordering between them) race and may return wrong indices.  Calls
 * queued on one stream are ordered and safe.
 */
#define WSP_ARGMAX_NO_ALLOC_MAX_GROUPS 65536
int wsp_argmax_no_alloc(const float* logits, const float* mask, uint32_t* indices, int row_count,
                        int row_length, void* stream);

#ifdef __cplusplus
}
#endif

#endif
