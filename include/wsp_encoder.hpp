/*
 * wsp_encoder.hpp -- the C++ binding of the audio front end, header only,
 * over the C ABI of wsp_encoder.h: Encoder (Lib/WhisperEACP/Encoder/
 * Encoder.h) with MelSpectrogram (Lib/WhisperEACP/Mel/MelSpectrogram.h) on
 * one CUDA device.  Status codes become the exceptions of wsp_decoder.hpp.
 */
#ifndef WSP_ENCODER_HPP
#define WSP_ENCODER_HPP

#include "wsp_decoder.hpp"
#include "wsp_encoder.h"

#include <cstdint>
#include <string>
#include <utility>
#include <vector>

namespace wsp {

using EncoderShape = wsp_encoder_shape;

class CudaEncoder {
public:
    CudaEncoder(const EncoderShape& shape, int device, wsp_dtype storage = WSP_FLOAT16) : shape_(shape) {
        check(wsp_encoder_create(&shape_, device, storage, &handle_));
    }
    ~CudaEncoder() { wsp_encoder_destroy(handle_); }
    CudaEncoder(const CudaEncoder&) = delete;
    CudaEncoder& operator=(const CudaEncoder&) = delete;
    CudaEncoder(CudaEncoder&& other) noexcept : shape_(other.shape_), handle_(std::exchange(other.handle_, nullptr)) {}

    const EncoderShape& shape() const { return shape_; }
    int positions() const { return (shape_.input_frames - 1) / 2 + 1; }

    /* One checkpoint tensor under its HuggingFace name (model.encoder.*). */
    void upload(const std::string& name, const void* data, wsp_dtype type, const std::vector<int64_t>& extents) {
        check(wsp_encoder_set_tensor(handle_, name.c_str(), type, extents.data(), (int)extents.size(), data));
    }
    /* The mel filterbank, [mel_bins][201] fp32. */
    void setFilters(const float* filters) { check(wsp_encoder_set_filters(handle_, filters)); }
    void checkWeights() const { check(wsp_encoder_check_weights(handle_)); }

    /* MelSpectrogram::encode: samples -> normalised log-mel [mel_bins][input_frames]. */
    std::vector<float> logMel(const float* samples, int count) {
        std::vector<float> mel((size_t)shape_.mel_bins * shape_.input_frames);
        check(wsp_encoder_log_mel(handle_, samples, count, mel.data()));
        return mel;
    }
    /* Encoder::encode: log-mel -> rows [positions][width] into `rows`. */
    void encode(const float* mel, float* rows) { check(wsp_encoder_encode(handle_, mel, rows)); }
    /* Samples -> rows [positions][width] into `rows`. */
    void encodeSamples(const float* samples, int count, float* rows) {
        check(wsp_encoder_encode_samples(handle_, samples, count, rows));
    }

private:
    EncoderShape shape_;
    wsp_encoder* handle_ = nullptr;
};

}  // namespace wsp

#endif
