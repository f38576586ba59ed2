/*
 * wsp_decoder.hpp -- the C++ binding of the B200 decoder token loop, header
 * only, over the C ABI of wsp_decoder.h (nothing else crosses into the
 * library).  It keeps the method names of WhisperEACP's Decoder
 * (Lib/WhisperEACP/Decoder/Decoder.h:49-127) and raises the reference's
 * exception types where a status code comes back: WSP_MODEL_ERROR as
 * wsp::ModelError (the role of WSP::ModelError, Model/ModelError.h:16),
 * WSP_LOGIC_ERROR as std::logic_error, WSP_INVALID_ARGUMENT as
 * std::invalid_argument, anything else as std::runtime_error.  Link with
 * -lwsp_b200.
 */
#ifndef WSP_DECODER_HPP
#define WSP_DECODER_HPP

#include "wsp_decoder.h"

#include <cstdint>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

namespace wsp {

struct ModelError : std::runtime_error {
    using std::runtime_error::runtime_error;
};

inline void check(int status) {
    if (status == WSP_OK) return;
    const std::string text = wsp_last_error();
    if (status == WSP_MODEL_ERROR) throw ModelError(text);
    if (status == WSP_LOGIC_ERROR) throw std::logic_error(text);
    if (status == WSP_INVALID_ARGUMENT) throw std::invalid_argument(text);
    throw std::runtime_error(text);
}

/* DecoderShape (Decoder/DecoderShape.h:20-31) under its C layout. */
using DecoderShape = wsp_decoder_shape;

/*
 * Decoder (Decoder.h:49-127) on one CUDA device: construction and prepare
 * are the constructor; `windows` independent windows decode in lockstep
 * (the reference's behaviour is windows == 1).
 */
class CudaDecoder {
public:
    CudaDecoder(const DecoderShape& shape, int device, int windows = 1, wsp_dtype storage = WSP_FLOAT16,
                int products = WSP_PRODUCTS_AUTO)
        : shape_(shape), windows_(windows) {
        check(wsp_decoder_create_products(&shape_, device, windows, storage, products, &handle_));
    }
    ~CudaDecoder() { wsp_decoder_destroy(handle_); }
    CudaDecoder(const CudaDecoder&) = delete;
    CudaDecoder& operator=(const CudaDecoder&) = delete;
    CudaDecoder(CudaDecoder&& other) noexcept
        : shape_(other.shape_), windows_(other.windows_), handle_(std::exchange(other.handle_, nullptr)) {}

    const DecoderShape& shape() const { return shape_; }
    int windows() const { return windows_; }

    /* One checkpoint tensor under its HuggingFace name (DecoderWeights,
       DecoderWeights.cpp:74-178); host data of the given element type. */
    void upload(const std::string& name, const void* data, wsp_dtype type, const std::vector<int64_t>& extents) {
        check(wsp_decoder_set_tensor(handle_, name.c_str(), type, extents.data(), (int)extents.size(), data));
    }
    void checkWeights() const { check(wsp_decoder_check_weights(handle_)); }

    /* Decoder::beginSequence: encoder rows fp32 [windows, cross_positions,
       width], host or device memory. */
    void beginSequence(const float* encoderOutput, int crossPositionCount = 0) {
        check(wsp_decoder_begin_sequence(handle_, encoderOutput, crossPositionCount));
    }

    /* Decoder::step for every window: tokens [windows, tokenCount]; logits
       [windows, tokenCount, vocabulary], hidden [windows, tokenCount, width]
       and argmax [windows, tokenCount] are optional outputs. */
    void step(const uint32_t* tokens, int tokenCount, float* logits, float* hidden = nullptr,
              uint32_t* argmax = nullptr) {
        check(wsp_decoder_step(handle_, tokens, tokenCount, logits, hidden, argmax));
    }

    int position() const {
        int p = 0;
        check(wsp_decoder_position(handle_, &p));
        return p;
    }
    int crossPositions() const {
        int c = 0;
        check(wsp_decoder_cross_positions(handle_, &c));
        return c;
    }

    /* Whisper::load's generation config (Whisper.cpp:148-254), once. */
    void setGeneration(const std::vector<uint32_t>& prompt, const std::vector<float>& firstMask,
                       const std::vector<float>& laterMask, int maximumTokens, uint32_t endOfText,
                       bool stopAtEndOfText = true) {
        prompt_length_ = (int)prompt.size();
        maximum_tokens_ = maximumTokens;
        const wsp_generation_config c{prompt.data(), (int32_t)prompt.size(),
                                      firstMask.empty() ? nullptr : firstMask.data(),
                                      laterMask.empty() ? nullptr : laterMask.data(), maximumTokens, endOfText,
                                      stopAtEndOfText ? 1 : 0};
        check(wsp_decoder_set_generation(handle_, &c));
    }

    /* Whisper::decodeTranscript (Whisper.cpp:1361-1449) for every window:
       each window's sampled ids, end-of-text excluded. */
    std::vector<std::vector<uint32_t>> decodeTranscript(const float* encoderOutput, int crossPositionCount = 0) {
        const int limit = stepLimit();
        std::vector<uint32_t> ids((size_t)windows_ * limit);
        std::vector<int32_t> counts((size_t)windows_);
        check(wsp_decoder_transcribe(handle_, encoderOutput, crossPositionCount, ids.data(), counts.data()));
        std::vector<std::vector<uint32_t>> out((size_t)windows_);
        for (int b = 0; b < windows_; ++b)
            out[b].assign(ids.begin() + (size_t)b * limit, ids.begin() + (size_t)b * limit + counts[b]);
        return out;
    }

    /* The step limit of Whisper.cpp:1375-1377. */
    int stepLimit() const {
        const int room = shape_.max_positions - prompt_length_ + 1;
        return maximum_tokens_ < room ? maximum_tokens_ : room;
    }

    wsp_decoder* handle() const { return handle_; }

private:
    DecoderShape shape_;
    int windows_;
    wsp_decoder* handle_ = nullptr;
    int prompt_length_ = 0;
    int maximum_tokens_ = 0;
};

}  // namespace wsp

#endif
