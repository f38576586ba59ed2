/*
 * wsp_encoder.h -- the C ABI of the B200 audio front end: the log-mel
 * spectrogram and the Whisper encoder, whose output rows are what
 * wsp_decoder_begin_sequence takes.  Same conventions as wsp_decoder.h
 * (status codes, wsp_last_error, host or device pointers, one device and
 * one host thread per object).
 *
 * Reference (paths within eyalamirmusic/WhisperEACP):
 *   MelSpectrogram (STFT, power, mel projection, log10, peak, normalise)
 *       Lib/WhisperEACP/Mel/MelSpectrogram.{h,cpp}, MelKernels.h:43-255
 *   Encoder (conv1d x2 + GELU, positional rows, pre-norm layers, final LN)
 *       Lib/WhisperEACP/Encoder/Encoder.cpp:69-175, EncoderShape.cpp
 *   EncoderWeights (HF names model.encoder.*)
 *       Lib/WhisperEACP/Encoder/EncoderWeights.{h,cpp}
 */
#ifndef WSP_ENCODER_H
#define WSP_ENCODER_H

#include "wsp_decoder.h"

#ifdef __cplusplus
extern "C" {
#endif

/* EncoderShape (Encoder/EncoderShape.h): input_frames mel frames (3000 for
   a 30 s window) become input_frames / 2 encoder positions (1500). */
typedef struct wsp_encoder_shape {
    int32_t mel_bins;           /* num_mel_bins: 80, or 128 for large-v3      */
    int32_t width;              /* d_model                                    */
    int32_t heads;              /* encoder_attention_heads (64-wide heads)    */
    int32_t layers;             /* encoder_layers                             */
    int32_t feed_forward_width; /* encoder_ffn_dim                            */
    int32_t input_frames;       /* 2 * max_source_positions                   */
} wsp_encoder_shape;

typedef struct wsp_encoder wsp_encoder;

/* Encoder::Encoder + prepare(device): weights are stored in `storage`
   (16-bit) for the tensor-core products; everything else stays fp32. */
int wsp_encoder_create(const wsp_encoder_shape* shape, int device, wsp_dtype storage, wsp_encoder** out);
void wsp_encoder_destroy(wsp_encoder* encoder);

/* One checkpoint tensor under its HuggingFace name (model.encoder.*), as
   EncoderWeights reads it; host data of the given element type. */
int wsp_encoder_set_tensor(wsp_encoder* encoder, const char* name, wsp_dtype dtype, const int64_t* extents,
                           int rank, const void* data);
/* The mel filterbank, [mel_bins][n_fft / 2 + 1] fp32 (preprocessor_config's
   mel_filters). */
int wsp_encoder_set_filters(wsp_encoder* encoder, const float* filters);
/* WSP_MODEL_ERROR naming the first tensor (or the filterbank) not set. */
int wsp_encoder_check_weights(const wsp_encoder* encoder);

/* MelSpectrogram::encode: `sample_count` 16 kHz samples (at most
   input_frames * 160; the rest of the window is silence) into the
   normalised log-mel [mel_bins][input_frames]. */
int wsp_encoder_log_mel(wsp_encoder* encoder, const float* samples, int sample_count, float* mel);

/* Encoder::encode: the log-mel [mel_bins][input_frames] into the encoder's
   output rows [input_frames / 2][width] fp32. */
int wsp_encoder_encode(wsp_encoder* encoder, const float* mel, float* rows);

/* Both: samples to encoder rows. */
int wsp_encoder_encode_samples(wsp_encoder* encoder, const float* samples, int sample_count, float* rows);

#ifdef __cplusplus
}
#endif

#endif
