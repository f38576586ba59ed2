// Host side of the B200 decoder: weights, caches, the step recording, the
// greedy search loop, and the C ABI of include/wsp_decoder.h.
//
// Reference (paths within eyalamirmusic/WhisperEACP):
//   Decoder / recordDecoderStep / recordSequenceStart  Lib/WhisperEACP/Decoder/Decoder.{h,cpp}
//   DecoderWeights                                     Lib/WhisperEACP/Decoder/DecoderWeights.{h,cpp}
//   greedy search                                      Lib/WhisperEACP/Whisper/Whisper.cpp:148-254,1158-1449
#include "../../include/wsp_decoder.h"
#include "host.h"
#include "cross_kv.cuh"
#include "kernels.cuh"
#include "schedule.h"
#include "step_launch.h"

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdlib>
#include <cmath>
#include <cstring>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

namespace wsp {

std::string& last_error_text() {
    thread_local std::string text;
    return text;
}

namespace {

bool is_device_pointer(const void* p) {
    cudaPointerAttributes attributes{};
    if (cudaPointerGetAttributes(&attributes, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return attributes.type == cudaMemoryTypeDevice || attributes.type == cudaMemoryTypeManaged;
}

uint16_t narrow(float v, Storage s) {
    if (s == Storage::f16) {
        __half h = __float2half_rn(v);
        uint16_t bits;
        std::memcpy(&bits, &h, 2);
        return bits;
    }
    __nv_bfloat16 h = __float2bfloat16_rn(v);
    uint16_t bits;
    std::memcpy(&bits, &h, 2);
    return bits;
}

float widen(const void* data, wsp_dtype dtype, size_t i) {
    if (dtype == WSP_FLOAT32) return static_cast<const float*>(data)[i];
    uint16_t bits = static_cast<const uint16_t*>(data)[i];
    if (dtype == WSP_FLOAT16) {
        __half h;
        std::memcpy(&h, &bits, 2);
        return __half2float(h);
    }
    __nv_bfloat16 h;
    std::memcpy(&h, &bits, 2);
    return __bfloat162float(h);
}

// ------------------------------------------------------------ tensors

// The per-layer names in the order DecoderLayerWeights declares them
// (DecoderWeights.h:25-51).
const char* const kLayerSuffixes[24] = {
    "self_attn_layer_norm.weight", "self_attn_layer_norm.bias",
    "self_attn.q_proj.weight", "self_attn.q_proj.bias", "self_attn.k_proj.weight",
    "self_attn.v_proj.weight", "self_attn.v_proj.bias",
    "self_attn.out_proj.weight", "self_attn.out_proj.bias",
    "encoder_attn_layer_norm.weight", "encoder_attn_layer_norm.bias",
    "encoder_attn.q_proj.weight", "encoder_attn.q_proj.bias", "encoder_attn.k_proj.weight",
    "encoder_attn.v_proj.weight", "encoder_attn.v_proj.bias",
    "encoder_attn.out_proj.weight", "encoder_attn.out_proj.bias",
    "final_layer_norm.weight", "final_layer_norm.bias",
    "fc1.weight", "fc1.bias", "fc2.weight", "fc2.bias"};

const char* const kGlobalNames[4] = {
    "model.decoder.embed_tokens.weight", "model.decoder.embed_positions.weight",
    "model.decoder.layer_norm.weight", "model.decoder.layer_norm.bias"};

struct LayerBuffers {
    DeviceBuffer ln1_w, ln1_b, qkv_w, qkv_b, o_w, o_b;
    DeviceBuffer ln2_w, ln2_b, qc_w, qc_b, vc_b, oc_w, oc_b;
    DeviceBuffer ln3_w, ln3_b, fc1_w, fc1_b, fc2_w, fc2_b;
};

class Decoder {
public:
    Decoder(const wsp_decoder_shape& shape, int device, int windows, Storage storage, int products)
        : shape_(shape), device_(device), windows_(windows), storage_(storage) {
        validate_shape();
        umma_ = choose_umma(products);
        CUDA_CHECK(cudaSetDevice(device_));
        CUDA_CHECK(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking));
        CUDA_CHECK(cudaDeviceGetAttribute(&sm_count_, cudaDevAttrMultiProcessorCount, device_));
        CUDA_CHECK(cudaDeviceGetAttribute(&max_shared_, cudaDevAttrMaxSharedMemoryPerBlockOptin, device_));
        for (cudaEvent_t& e : phase_events_) CUDA_CHECK(cudaEventCreate(&e));
        allocate_weights();
        allocate_state();
        ensure_row_capacity(4);
    }

    ~Decoder() {
        cudaSetDevice(device_);
        for (cudaEvent_t e : phase_events_)
            if (e) cudaEventDestroy(e);
        if (stream_) cudaStreamDestroy(stream_);
    }

    // ---------------------------------------------------------------- weights

    void set_tensor(const char* name_c, wsp_dtype dtype, const int64_t* extents, int rank, const void* data) {
        if (name_c == nullptr || data == nullptr || (rank > 0 && extents == nullptr))
            throw InvalidArgument("set_tensor needs a name, extents and data");
        if (dtype != WSP_FLOAT32 && dtype != WSP_FLOAT16 && dtype != WSP_BFLOAT16)
            throw InvalidArgument("tensor element type must be float32, float16 or bfloat16");
        const std::string name(name_c);
        if (name.rfind("model.decoder.", 0) != 0) return;  // the encoder's, and anything else
        CUDA_CHECK(cudaSetDevice(device_));
        const int d = shape_.width, f = shape_.feed_forward_width;

        int global = -1;
        for (int i = 0; i < 4; ++i)
            if (name == kGlobalNames[i]) global = i;
        if (global >= 0) {
            if (global == 0) {
                require_extents(name, extents, rank, {shape_.vocabulary_size, d});
                audit_narrowing(name, dtype, data, (size_t)shape_.vocabulary_size * d);
                // The layout of the logits' products (fragment-packed, or the
                // tcgen05 tiles); the embedding gathers from the same table.
                if (umma_)
                    patch16(token_table_, shape_.vocabulary_size, d, dtype, data,
                            [&](int r, int c) { return weight_offset(r, c, padded(d)); });
                else
                    upload_packed(token_table_, 0, shape_.vocabulary_size, d, padded(d), dtype, data);
            } else if (global == 1) {
                // A model may carry more positions than a run needs; fewer is an error.
                if (rank != 2 || extents[1] != d || extents[0] < shape_.max_positions)
                    throw ModelError(name + " has shape " + describe(extents, rank) + ", expected [>=" +
                                     std::to_string(shape_.max_positions) + ", " + std::to_string(d) + "]");
                upload_floats(position_table_, 0, (size_t)shape_.max_positions * d, dtype, data);
            } else {
                require_extents(name, extents, rank, {d});
                upload_floats(global == 2 ? final_w_ : final_b_, 0, d, dtype, data);
            }
            present_[global] = true;
            return;
        }

        const std::string prefix = "model.decoder.layers.";
        if (name.rfind(prefix, 0) != 0) throw ModelError("unknown decoder tensor " + name);
        size_t dot = name.find('.', prefix.size());
        if (dot == std::string::npos) throw ModelError("unknown decoder tensor " + name);
        int layer = -1;
        try {
            layer = std::stoi(name.substr(prefix.size(), dot - prefix.size()));
        } catch (...) {
            throw ModelError("unknown decoder tensor " + name);
        }
        if (layer < 0 || layer >= shape_.layers)
            throw ModelError(name + " names layer " + std::to_string(layer) + " of a " +
                             std::to_string(shape_.layers) + "-layer decoder");
        const std::string suffix = name.substr(dot + 1);
        int which = -1;
        for (int i = 0; i < 24; ++i)
            if (suffix == kLayerSuffixes[i]) which = i;
        if (which < 0) throw ModelError("unknown decoder tensor " + name);

        LayerBuffers& L = layers_[layer];
        const int kpd = padded(d), kpf = padded(f);
        // The projection matrices are narrowed to the storage type.
        static const bool kNarrowed[24] = {false, false, true,  false, true,  true,  false, true,
                                           false, false, false, true,  false, true,  true,  false,
                                           true,  false, false, false, true,  false, true,  false};
        if (kNarrowed[which]) {
            size_t count = 1;
            for (int i = 0; i < rank; ++i) count *= (size_t)std::max<int64_t>(extents[i], 0);
            if (which == 20 || which == 22) require_extents(name, extents, rank, which == 20 ? std::initializer_list<int>{f, d} : std::initializer_list<int>{d, f});
            else require_extents(name, extents, rank, {d, d});
            audit_narrowing(name, dtype, data, count);
        }
        switch (which) {
        case 0: require_extents(name, extents, rank, {d}); upload_floats(L.ln1_w, 0, d, dtype, data); break;
        case 1: require_extents(name, extents, rank, {d}); upload_floats(L.ln1_b, 0, d, dtype, data); break;
        case 2: require_extents(name, extents, rank, {d, d}); patch_qkv(L.qkv_w, 0, dtype, data); break;
        case 3:
            require_extents(name, extents, rank, {d});
            patch_floats(L.qkv_b, d, dtype, data, [&](int i) { return qkv_row(0, i); });
            break;
        case 4: require_extents(name, extents, rank, {d, d}); patch_qkv(L.qkv_w, 1, dtype, data); break;
        case 5: require_extents(name, extents, rank, {d, d}); patch_qkv(L.qkv_w, 2, dtype, data); break;
        case 6:
            require_extents(name, extents, rank, {d});
            patch_floats(L.qkv_b, d, dtype, data, [&](int i) { return qkv_row(2, i); });
            break;
        case 7:
            require_extents(name, extents, rank, {d, d});
            patch16(L.o_w, d, d, dtype, data, [&](int r, int c) { return weight_offset(r, c, kpd); });
            break;
        case 8: require_extents(name, extents, rank, {d}); upload_floats(L.o_b, 0, d, dtype, data); break;
        case 9: require_extents(name, extents, rank, {d}); upload_floats(L.ln2_w, 0, d, dtype, data); break;
        case 10: require_extents(name, extents, rank, {d}); upload_floats(L.ln2_b, 0, d, dtype, data); break;
        case 11:
            require_extents(name, extents, rank, {d, d});
            patch16(L.qc_w, d, d, dtype, data, [&](int r, int c) { return weight_offset(q_row(r), c, kpd); });
            break;
        case 12:
            require_extents(name, extents, rank, {d});
            patch_floats(L.qc_b, d, dtype, data, [&](int i) { return q_row(i); });
            break;
        case 13:  // cross keys and values: head h of layer l is rows [K_h; V_h]
        case 14:
            require_extents(name, extents, rank, {d, d});
            upload_cross_projection(layer, which == 14 ? 1 : 0, dtype, data);
            break;
        case 15: require_extents(name, extents, rank, {d}); upload_floats(L.vc_b, 0, d, dtype, data); break;
        case 16:
            require_extents(name, extents, rank, {d, d});
            patch16(L.oc_w, d, d, dtype, data, [&](int r, int c) { return weight_offset(r, c, kpd); });
            break;
        case 17: require_extents(name, extents, rank, {d}); upload_floats(L.oc_b, 0, d, dtype, data); break;
        case 18: require_extents(name, extents, rank, {d}); upload_floats(L.ln3_w, 0, d, dtype, data); break;
        case 19: require_extents(name, extents, rank, {d}); upload_floats(L.ln3_b, 0, d, dtype, data); break;
        case 20:
            require_extents(name, extents, rank, {f, d});
            patch16(L.fc1_w, f, d, dtype, data, [&](int r, int c) { return weight_offset(r, c, kpd); });
            break;
        case 21: require_extents(name, extents, rank, {f}); upload_floats(L.fc1_b, 0, f, dtype, data); break;
        case 22:
            require_extents(name, extents, rank, {d, f});
            patch16(L.fc2_w, d, f, dtype, data, [&](int r, int c) { return weight_offset(r, c, kpf); });
            break;
        case 23: require_extents(name, extents, rank, {d}); upload_floats(L.fc2_b, 0, d, dtype, data); break;
        }
        present_[4 + 24 * layer + which] = true;
    }

    void check_weights() const {
        for (int i = 0; i < 4; ++i)
            if (!present_[i]) throw ModelError(std::string("the decoder has no tensor ") + kGlobalNames[i]);
        for (int l = 0; l < shape_.layers; ++l)
            for (int i = 0; i < 24; ++i)
                if (!present_[4 + 24 * l + i])
                    throw ModelError("the decoder has no tensor model.decoder.layers." + std::to_string(l) + "." +
                                     kLayerSuffixes[i]);
    }

    // ------------------------------------------------------------ sequences

    // Decoder::beginSequence (Decoder.cpp:229-268).
    void begin_sequence(const float* encoder_rows, int cross_positions) {
        if (encoder_rows == nullptr) throw InvalidArgument("begin_sequence needs encoder rows");
        if (cross_positions < 0 || cross_positions > shape_.cross_positions)
            throw ModelError("a decoder built for " + std::to_string(shape_.cross_positions) +
                             " encoder rows was asked to attend to " + std::to_string(cross_positions));
        check_weights();
        CUDA_CHECK(cudaSetDevice(device_));
        const int rows = cross_positions == 0 ? shape_.cross_positions : cross_positions;
        const size_t elements = (size_t)windows_ * shape_.cross_positions * shape_.width;
        const float* source = encoder_rows;
        // Host rows, or device rows the kernel cannot read as float4s, go
        // through the staging buffer.
        if (!is_device_pointer(encoder_rows) || reinterpret_cast<uintptr_t>(encoder_rows) % 16 != 0) {
            CUDA_CHECK(cudaMemcpyAsync(encoder_staging_.get(), encoder_rows, elements * sizeof(float),
                                       cudaMemcpyDefault, stream_));
            source = encoder_staging_.get<float>();
        }
        if (cross_weights_dirty_) {
            CUDA_CHECK(cudaMemcpy(cross_kv_w_.get(), cross_kv_host_.data(), cross_kv_host_.size() * 2,
                                  cudaMemcpyHostToDevice));
            settle_legacy_stream();
            cross_weights_dirty_ = false;
        }

        // recordSequenceStart (Decoder.cpp:121-146): every layer's cross keys
        // and values for every window in one tcgen05 launch (cross_kv.cuh),
        // written as the cache layout [layer][window][head][X][K | V].  The
        // value bias is added after the attention instead (the weights sum
        // to one).
        const int d = shape_.width, D = d / shape_.heads;
        CrossKvArgs args{};
        args.encoder = source;
        args.weight = cross_kv_w_.get();
        args.out = cross_kv_.get();
        args.windows = windows_;
        args.rows = rows;
        args.row_stride = shape_.cross_positions;
        args.width = d;
        args.kblocks = (d + kCrossBlockCols - 1) / kCrossBlockCols;
        args.columns = 2 * d * shape_.layers;
        args.head_width = D;
        args.groups = shape_.layers * shape_.heads;
        args.heads = shape_.heads;
        args.status = state_.get<int>() + kCrossStatusWord;
        CUDA_CHECK(cudaMemsetAsync(args.status, 0, sizeof(int), stream_));
        try {
            launch_cross_kv(storage_ == Storage::f16, args, sm_count_, stream_);
        } catch (const std::runtime_error& e) {
            throw CudaFailure(e.what(), false);
        }
        ++launches_;
        CUDA_CHECK(cudaMemsetAsync(state_.get(), 0, kStateWords * sizeof(int), stream_));
        CUDA_CHECK(cudaGetLastError());
        active_cross_ = rows;
        position_ = 0;
        started_ = true;
    }

    // Decoder::step (Decoder.cpp:270-308) for every window, teacher-forced.
    void step(const uint32_t* tokens, int count, float* logits, float* hidden, uint32_t* argmax) {
        if (!started_) throw LogicError("a decoder step needs a sequence: call begin_sequence first");
        if (count <= 0) throw ModelError("a decoder step needs at least one token");
        if (tokens == nullptr) throw InvalidArgument("a decoder step needs its tokens");
        if (position_ + count > shape_.max_positions)
            throw ModelError("this step would carry the sequence to " + std::to_string(position_ + count) +
                             " tokens, past the " + std::to_string(shape_.max_positions) +
                             " this decoder was built for");
        CUDA_CHECK(cudaSetDevice(device_));
        std::vector<uint32_t> ids((size_t)windows_ * count);
        if (is_device_pointer(tokens))
            CUDA_CHECK(cudaMemcpy(ids.data(), tokens, ids.size() * 4, cudaMemcpyDeviceToHost));
        else
            std::memcpy(ids.data(), tokens, ids.size() * 4);
        for (uint32_t id : ids)
            if (id >= (uint32_t)shape_.vocabulary_size)
                throw ModelError("token " + std::to_string(id) + " is outside the " +
                                 std::to_string(shape_.vocabulary_size) + "-token vocabulary");
        ensure_row_capacity(count);
        const int R = windows_ * count;
        // The ids go into the ring slots the step embeds.
        CUDA_CHECK(cudaMemcpy2DAsync(ring_.get<uint32_t>() + position_, ring_stride() * 4, ids.data(), count * 4,
                                     count * 4, windows_, cudaMemcpyHostToDevice, stream_));
        const bool logits_on_device = logits && is_device_pointer(logits);
        const bool hidden_on_device = hidden && is_device_pointer(hidden);
        if (logits && !logits_on_device) ensure_staging(logits_staging_, (size_t)R * shape_.vocabulary_size * 4);
        if (hidden && !hidden_on_device) ensure_staging(hidden_staging_, (size_t)R * shape_.width * 4);
        float* logits_dev = logits ? (logits_on_device ? logits : logits_staging_.get<float>()) : nullptr;
        float* hidden_dev = hidden ? (hidden_on_device ? hidden : hidden_staging_.get<float>()) : nullptr;
        launch_steps(count, /*sample=*/false, nullptr, logits_dev, hidden_dev, row_tokens_.get<uint32_t>(), 1,
                     /*stop=*/false, nullptr);
        if (logits && !logits_on_device)
            CUDA_CHECK(cudaMemcpyAsync(logits, logits_dev, (size_t)R * shape_.vocabulary_size * 4,
                                       cudaMemcpyDeviceToHost, stream_));
        if (hidden && !hidden_on_device)
            CUDA_CHECK(cudaMemcpyAsync(hidden, hidden_dev, (size_t)R * shape_.width * 4, cudaMemcpyDeviceToHost,
                                       stream_));
        if (argmax)
            CUDA_CHECK(cudaMemcpyAsync(argmax, row_tokens_.get(), (size_t)R * 4, cudaMemcpyDefault, stream_));
        CUDA_CHECK(cudaStreamSynchronize(stream_));
        check_device_errors();
        position_ += count;
    }

    int position() const { return position_; }
    int cross_positions() const { return active_cross_; }

    // ---------------------------------------------------------- greedy search

    void set_generation(const wsp_generation_config& c) {
        if (c.prompt == nullptr || c.prompt_length <= 0) throw ModelError("the prompt needs at least one token");
        if (c.prompt_length >= shape_.max_positions)
            throw ModelError("a prompt of " + std::to_string(c.prompt_length) + " tokens leaves no room in a " +
                             std::to_string(shape_.max_positions) + "-position window");
        if (c.maximum_tokens <= 0) throw ModelError("a transcript has to be allowed at least one token");
        for (int i = 0; i < c.prompt_length; ++i)
            if (c.prompt[i] >= (uint32_t)shape_.vocabulary_size)
                throw ModelError("prompt token " + std::to_string(c.prompt[i]) + " is outside the vocabulary");
        CUDA_CHECK(cudaSetDevice(device_));
        // A transcription still queued (enqueue_transcribe without its read)
        // reads the masks and the prompt ring from the device: let it finish
        // before they are overwritten.
        CUDA_CHECK(cudaStreamSynchronize(stream_));
        prompt_.assign(c.prompt, c.prompt + c.prompt_length);
        maximum_tokens_ = c.maximum_tokens;
        end_of_text_ = c.end_of_text;
        stop_at_end_of_text_ = c.stop_at_end_of_text != 0;
        const size_t v = shape_.vocabulary_size;
        std::vector<float> masks(2 * v, 0.f);
        if (c.first_step_mask) copy_floats(masks.data(), c.first_step_mask, v);
        if (c.later_step_mask) copy_floats(masks.data() + v, c.later_step_mask, v);
        CUDA_CHECK(cudaMemcpy(masks_.get(), masks.data(), masks.size() * 4, cudaMemcpyHostToDevice));
        std::vector<uint32_t> ring_prompt((size_t)windows_ * ring_stride(), 0u);
        for (int b = 0; b < windows_; ++b)
            std::copy(prompt_.begin(), prompt_.end(), ring_prompt.begin() + (size_t)b * ring_stride());
        CUDA_CHECK(cudaMemcpy(ring_prompt_.get(), ring_prompt.data(), ring_prompt.size() * 4, cudaMemcpyHostToDevice));
        settle_legacy_stream();
        ensure_row_capacity((int)prompt_.size());
        generation_set_ = true;
    }

    int step_limit() const {
        // Whisper.cpp:1375-1377
        return std::min(maximum_tokens_, shape_.max_positions - (int)prompt_.size() + 1);
    }

    // encodeStep for step 0 (Whisper.cpp:1190-1205): sequence start, the
    // prompt in one step, sampling under the first-step mask.
    void enqueue_start(const float* encoder_rows, int cross_positions) {
        if (!generation_set_) throw LogicError("set the generation config before transcribing");
        CUDA_CHECK(cudaEventRecord(phase_events_[0], stream_));
        begin_sequence(encoder_rows, cross_positions);
        CUDA_CHECK(cudaEventRecord(phase_events_[1], stream_));
        CUDA_CHECK(cudaMemcpyAsync(ring_.get(), ring_prompt_.get(), ring_prompt_.bytes(), cudaMemcpyDeviceToDevice,
                                   stream_));
        CUDA_CHECK(cudaMemsetAsync(ended_.get(), 0, ended_.bytes(), stream_));
        ensure_row_capacity((int)prompt_.size());
        launch_steps((int)prompt_.size(), /*sample=*/true, masks_.get<float>(), nullptr, nullptr, nullptr, 1,
                     stop_at_end_of_text_, nullptr);
        CUDA_CHECK(cudaEventRecord(phase_events_[2], stream_));
        CUDA_CHECK(cudaEventRecord(phase_events_[3], stream_));
        position_ = (int)prompt_.size();
        sampled_steps_ = 1;
        queued_steps_ = 0;
    }

    // encodeStep for steps k > 0 (Whisper.cpp:1207-1212): `steps` single-token
    // steps in one launch of the decode kernel, each sampling into the slot
    // the next one embeds.
    void enqueue_steps(int steps) {
        if (steps <= 0) return;
        if (position_ + steps > shape_.max_positions) throw ModelError("the window is full");
        launch_steps(1, /*sample=*/true, masks_.get<float>() + shape_.vocabulary_size, nullptr, nullptr, nullptr,
                     steps, stop_at_end_of_text_, nullptr);
        CUDA_CHECK(cudaEventRecord(phase_events_[3], stream_));
        position_ += steps;
        queued_steps_ += steps;
    }

    void enqueue_transcribe(const float* encoder_rows, int cross_positions, int steps) {
        if (steps <= 0 || steps > step_limit())
            throw ModelError("asked for " + std::to_string(steps) + " steps; the limit is " +
                             std::to_string(step_limit()));
        enqueue_start(encoder_rows, cross_positions);
        enqueue_steps(steps - 1);
    }

    void read_transcript(uint32_t* tokens, int32_t* counts) {
        CUDA_CHECK(cudaSetDevice(device_));
        CUDA_CHECK(cudaStreamSynchronize(stream_));
        check_device_errors();
        int state[kStateWords];
        CUDA_CHECK(cudaMemcpy(state, state_.get(), sizeof state, cudaMemcpyDeviceToHost));
        if (queued_steps_ > 0) {
            // With the stop enabled the kernel returns once every window has
            // ended; the steps it ran are the ones sampled.
            const int ran = state[kStepsDone];
            sampled_steps_ += ran;
            position_ -= queued_steps_ - ran;
            queued_steps_ = 0;
        }
        const int steps = sampled_steps_;
        const int p = (int)prompt_.size();
        std::vector<uint32_t> ring((size_t)windows_ * ring_stride());
        CUDA_CHECK(cudaMemcpy(ring.data(), ring_.get(), ring.size() * 4, cudaMemcpyDeviceToHost));
        for (int b = 0; b < windows_; ++b) {
            int count = 0;
            for (int k = 0; k < steps; ++k) {
                const uint32_t id = ring[(size_t)b * ring_stride() + p + k];
                if (stop_at_end_of_text_ && id == end_of_text_) break;
                if (tokens) tokens[(size_t)b * step_limit() + k] = id;
                ++count;
            }
            if (counts) counts[b] = count;
        }
    }

    // Whisper::decodeTranscript (Whisper.cpp:1361-1449): the prompt step,
    // then every later step in one launch that stops by itself once every
    // window has sampled end-of-text (with stop_at_end_of_text).
    void transcribe(const float* encoder_rows, int cross_positions, uint32_t* tokens, int32_t* counts) {
        const int limit = step_limit();
        enqueue_start(encoder_rows, cross_positions);
        enqueue_steps(limit - 1);
        read_transcript(tokens, counts);
    }

    cudaStream_t stream() const { return stream_; }

    void synchronize() {
        CUDA_CHECK(cudaSetDevice(device_));
        CUDA_CHECK(cudaStreamSynchronize(stream_));
        check_device_errors();
    }

    // Per-op timing of single-token sampled steps: the decode kernel stamps
    // %globaltimer after each op's grid barrier; one launch per step.
    void time_kernels(int steps, float* ms, int* launches) {
        if (!generation_set_ || !started_) throw LogicError("time_kernels needs a transcription in progress");
        if (position_ + steps > shape_.max_positions) throw ModelError("not enough room left in the window");
        CUDA_CHECK(cudaSetDevice(device_));
        std::vector<double> total(WSP_KERNEL_CLASSES, 0.0);
        std::vector<int> count(WSP_KERNEL_CLASSES, 0);
        std::vector<unsigned long long> stamps;
        std::vector<unsigned long long> sections(kTraceSections, 0);
        trace_cycles_.assign(kTraceSections, 0.0);
        for (int i = 0; i < steps; ++i) {
            CUDA_CHECK(cudaMemsetAsync(profile_.get<unsigned long long>() + kTraceOffset, 0,
                                       kTraceSections * sizeof(unsigned long long), stream_));
            const std::vector<StepOp>& ops = launch_steps(1, true, masks_.get<float>() + shape_.vocabulary_size,
                                                          nullptr, nullptr, nullptr, 1, false,
                                                          profile_.get<unsigned long long>());
            stamps.resize(ops.size() + 1);
            CUDA_CHECK(cudaMemcpyAsync(stamps.data(), profile_.get(), stamps.size() * 8, cudaMemcpyDeviceToHost,
                                       stream_));
            CUDA_CHECK(cudaMemcpyAsync(sections.data(), profile_.get<unsigned long long>() + kTraceOffset,
                                       kTraceSections * sizeof(unsigned long long), cudaMemcpyDeviceToHost, stream_));
            CUDA_CHECK(cudaStreamSynchronize(stream_));
            for (int t = 0; t < kTraceSections; ++t) trace_cycles_[t] += (double)sections[t] / steps;
            if (i == 0) op_us_.assign(ops.size(), 0.0);
            op_kinds_.resize(ops.size());
            for (size_t o = 0; o < ops.size(); ++o) {
                const int cls = op_class(ops[o].kind);
                total[cls] += (stamps[o + 1] - stamps[o]) * 1e-6;
                count[cls] += 1;
                op_kinds_[o] = ops[o].kind;
                if (o < op_us_.size()) op_us_[o] += (stamps[o + 1] - stamps[o]) * 1e-3 / steps;
            }
            ++position_;
        }
        check_device_errors();
        for (int c = 0; c < WSP_KERNEL_CLASSES; ++c) {
            if (ms) ms[c] = count[c] ? (float)(total[c] / count[c]) : 0.f;
            if (launches) launches[c] = steps ? count[c] / steps : 0;
        }
    }

    // Mean microseconds of one grid barrier of the decode kernel: a launch
    // whose op list is `count` empty ops, stamped after each barrier.
    float time_barriers(int count) {
        CUDA_CHECK(cudaSetDevice(device_));
        if (count <= 0 || count + 1 > 8 * shape_.layers + 8) throw InvalidArgument("barrier count out of range");
        std::vector<StepOp> ops(count);
        for (auto& o : ops) o.kind = kOpNone;
        if (ops_probe_dev_.bytes() < ops.size() * sizeof(StepOp)) ops_probe_dev_.allocate(ops.size() * sizeof(StepOp));
        CUDA_CHECK(cudaMemcpy(ops_probe_dev_.get(), ops.data(), ops.size() * sizeof(StepOp), cudaMemcpyHostToDevice));
        settle_legacy_stream();
        StepParams p = base_params(1, true, nullptr, nullptr, nullptr, nullptr, 1, false);
        p.profile = profile_.get<unsigned long long>();
        p.ops = ops_probe_dev_.get<StepOp>();
        p.n_ops = count;
        p.steps = 1;
        const bool half = storage_ == Storage::f16;
        configure_stream(half, p);
        const int blocks = decode_blocks_per_sm(half, p, kMaxCrossChunk);
        if (blocks <= 0) throw CudaFailure("the decode kernel does not fit on an SM", false);
        upload_schedule(p, ops, sm_count_ * std::min(blocks, kMaxBlocksPerSm));
        CUDA_CHECK(cudaMemsetAsync(state_.get<int>() + kAbort, 0, 2 * sizeof(int), stream_));
        CUDA_CHECK(cudaMemsetAsync(barrier_.get(), 0, barrier_.bytes(), stream_));
        launch_decode(half, p, kMaxCrossChunk, sm_count_ * std::min(blocks, kMaxBlocksPerSm), stream_);
        std::vector<unsigned long long> stamps(count + 1);
        CUDA_CHECK(cudaMemcpyAsync(stamps.data(), profile_.get(), stamps.size() * 8, cudaMemcpyDeviceToHost, stream_));
        CUDA_CHECK(cudaStreamSynchronize(stream_));
        check_device_errors();
        // The first barrier also absorbs the launch's start-up skew.
        return count > 1 ? (float)((stamps[count] - stamps[1]) * 1e-3 / (count - 1)) : 0.f;
    }

    // Microseconds of each op of the step (its work and the grid barrier
    // after it) and its kind, averaged over the last time_kernels run.
    int op_times(float* us, int* kinds, int capacity) const {
        for (int i = 0; i < capacity && i < (int)op_us_.size(); ++i) {
            if (us) us[i] = (float)op_us_[i];
            if (kinds) kinds[i] = op_kinds_[i];
        }
        return (int)op_us_.size();
    }

    // Section cycles of CTA 0 per step, from the last time_kernels run.
    void trace_cycles(double* out, int count) const {
        for (int i = 0; i < count; ++i) out[i] = i < (int)trace_cycles_.size() ? trace_cycles_[i] : 0.0;
    }

    // Milliseconds of the last transcription's phases, from CUDA events on
    // the decoder's stream: the sequence start (encoder-row narrowing and the
    // cross K/V product), the prompt step's launch, and the launch that runs
    // every later step (0 when there was none).
    void phase_ms(float* ms) {
        CUDA_CHECK(cudaSetDevice(device_));
        CUDA_CHECK(cudaEventSynchronize(phase_events_[3]));
        for (int i = 0; i < 3; ++i) CUDA_CHECK(cudaEventElapsedTime(ms + i, phase_events_[i], phase_events_[i + 1]));
    }

    // Kernel launches of this library per transcription: the cross key/value
    // projection, the prompt step, and the launch that runs every later step.
    int step_launches() const { return 3; }

private:
    int ring_stride() const { return shape_.max_positions + 1; }

    void validate_shape() {
        const auto& s = shape_;
        if (s.width <= 0 || s.heads <= 0 || s.layers <= 0 || s.feed_forward_width <= 0 || s.vocabulary_size <= 0 ||
            s.max_positions <= 0 || s.cross_positions <= 0 || windows_ <= 0)
            throw ModelError("every decoder extent and the window count must be positive");
        if (s.width % s.heads != 0) throw ModelError("the width must be a whole number of heads");
        const int D = s.width / s.heads;
        if (D > 64 || D % 4 != 0)
            throw ModelError("heads must be at most 64 wide and a multiple of 4 (SingleQueryAttention.cpp:37-45)");
        if (s.width > 1536) throw ModelError("widths above 1536 are not supported");
        if (storage_ != Storage::f16 && storage_ != Storage::bf16)
            throw InvalidArgument("storage must be float16 or bfloat16");
    }

    static size_t round16(size_t n) { return (n + 15) / 16 * 16; }

    // The products' form.  tcgen05 tiles (128 weight rows against every
    // window's row, accumulated in tensor memory) need widths in 64-column
    // blocks, 64-wide heads and at least 16 windows (an MMA's N >= 16).
    // With the activations' hi and lo planes, measured on B200 they beat the
    // mma.sync tiles from 32 windows (small.en at 32 windows: 10.3 us a
    // product against 13.2; medium.en at 64: 12.7 against 20.4), so AUTO
    // picks them from kUmmaWindows windows.
    static constexpr int kUmmaWindows = 32;
    bool umma_possible() const {
        return windows_ >= 16 && shape_.width % 64 == 0 && shape_.feed_forward_width % 64 == 0 && head_width() == 64;
    }
    bool choose_umma(int products) const {
        if (products == WSP_PRODUCTS_MMA) return false;
        if (products == WSP_PRODUCTS_TCGEN05) {
            if (!umma_possible())
                throw ModelError("tcgen05 products need widths in 64-column blocks, 64-wide heads and 16+ windows");
            return true;
        }
        return umma_possible() && windows_ >= kUmmaWindows;
    }
    // Rows a product weight matrix is allocated with: whole 16-row tiles, or
    // whole 128-row tiles for the tensor-core products.
    size_t weight_rows(size_t n) const { return umma_ ? (n + 127) / 128 * 128 : round16(n); }
    // Element offset of (row n, column k) of a product weight with inner size kp.
    size_t weight_offset(int n, int k, int kp) const {
        return umma_ ? umma_offset(n, k, kp / 64) : packed_offset(n, k, kp / 32);
    }
    // Rows of an activation buffer: whole 16-row groups (a tensor-core item's
    // rows round up to 16) of every row a step can hold.
    int act_rows() const { return (windows_ * token_capacity_ + 15) / 16 * 16; }

    int head_width() const { return shape_.width / shape_.heads; }
    // Packed row of the q (0), k (1) or v (2) row i of a head-grouped q/k/v
    // matrix: head h owns rows [h*G, h*G + 3D), G = 3D rounded to a tile.
    int qkv_row(int which, int i) const {
        const int D = head_width();
        return (i / D) * (int)round16(3 * D) + which * D + i % D;
    }
    // Packed row of cross q row i: head h owns rows [h*G, h*G + D), G = D rounded.
    int q_row(int i) const {
        const int D = head_width();
        return (i / D) * (int)round16(D) + i % D;
    }

    void allocate_weights() {
        const size_t d = shape_.width, f = shape_.feed_forward_width, L = shape_.layers;
        const size_t H = shape_.heads, D = d / H;
        const size_t kpd = padded(d), kpf = padded(f);
        token_table_.allocate(weight_rows(shape_.vocabulary_size) * kpd * 2);
        position_table_.allocate((size_t)shape_.max_positions * d * 4);
        final_w_.allocate(d * 4);
        final_b_.allocate(d * 4);
        cross_kv_host_.assign(cross_weight_elements(), 0);
        cross_kv_w_.allocate(cross_kv_host_.size() * 2);
        layers_.reset(new LayerBuffers[L]);
        for (size_t i = 0; i < L; ++i) {
            LayerBuffers& l = layers_[i];
            l.ln1_w.allocate(d * 4); l.ln1_b.allocate(d * 4);
            l.qkv_w.allocate(weight_rows(H * round16(3 * D)) * kpd * 2); l.qkv_b.allocate(H * round16(3 * D) * 4);
            l.o_w.allocate(weight_rows(d) * kpd * 2); l.o_b.allocate(d * 4);
            l.ln2_w.allocate(d * 4); l.ln2_b.allocate(d * 4);
            l.qc_w.allocate(weight_rows(H * round16(D)) * kpd * 2); l.qc_b.allocate(H * round16(D) * 4);
            l.vc_b.allocate(d * 4);
            l.oc_w.allocate(weight_rows(d) * kpd * 2); l.oc_b.allocate(d * 4);
            l.ln3_w.allocate(d * 4); l.ln3_b.allocate(d * 4);
            l.fc1_w.allocate(weight_rows(f) * kpd * 2); l.fc1_b.allocate(f * 4);
            l.fc2_w.allocate(weight_rows(d) * kpf * 2); l.fc2_b.allocate(d * 4);
        }
        present_.assign(4 + 24 * L, false);
    }

    void allocate_state() {
        const size_t d = shape_.width, L = shape_.layers, B = windows_;
        const size_t X = shape_.cross_positions, P = shape_.max_positions;
        self_keys_.allocate(L * B * P * d * 2);
        self_values_.allocate(L * B * P * d * 2);
        cross_kv_.allocate(B * X * 2 * d * L * 2);
        encoder_staging_.allocate(B * X * d * 4);
        ring_.allocate(B * ring_stride() * 4);
        ring_prompt_.allocate(B * ring_stride() * 4);
        state_.allocate((kCrossStatusWord + 1) * sizeof(int));
        barrier_.allocate(64);
        ended_.allocate((size_t)windows_);
        profile_.allocate(1024 * sizeof(unsigned long long));
        masks_.allocate(2 * (size_t)shape_.vocabulary_size * 4);
    }


    void ensure_row_capacity(int tokens) {
        if (tokens <= token_capacity_) return;
        token_capacity_ = std::max(tokens, token_capacity_);
        const size_t R = (size_t)windows_ * token_capacity_;
        const size_t d = shape_.width, f = shape_.feed_forward_width, H = shape_.heads, D = d / H;
        hidden_.allocate(R * d * 4);
        queries_.allocate(R * d * 4);
        // 16-bit activations a product reads: a hi plane and a lo plane.
        const size_t A = (R + 15) / 16 * 16;
        normalised_.allocate(2 * A * padded(d) * 2);
        attended_.allocate(2 * A * padded(d) * 2);
        feed_forward_.allocate(2 * A * padded(f) * 2);
        partial_.allocate(R * H * kMaxCrossSplits * (D + 2) * 4);
        // Fused out-projections (a few rows): the heads' partial rows of the
        // self and the cross attention, and the residual rows between them.
        const size_t Rf = std::min<size_t>(R, kInlineNormRows);
        out_partials_.allocate(2 * H * Rf * d * 4);
        hidden_mid_.allocate(Rf * d * 4);
        hidden_alt_.allocate(Rf * d * 4);
        ffn_partials_.allocate((size_t)kFfnParts * Rf * d * 4);
        const size_t grid = (size_t)kMaxBlocksPerSm * sm_count_;
        candidate_values_.allocate(R * grid * 4);
        candidate_indices_.allocate(R * grid * 4);
        row_tokens_.allocate(R * 4);
        counters_.allocate((R * H + 1) * sizeof(unsigned));
    }

    void ensure_staging(DeviceBuffer& buffer, size_t bytes) {
        if (buffer.bytes() < bytes) buffer.allocate(bytes);
    }

    void check_device_errors() {
        int state[kCrossStatusWord + 1];
        CUDA_CHECK(cudaMemcpy(state, state_.get(), sizeof state, cudaMemcpyDeviceToHost));
        if (state[kCrossStatusWord] != 0) {
            static const char* const kinds[] = {"?", "encoder rows", "weights", "a free stage", "a free accumulator",
                                                "its products to drain", "an accumulator"};
            const int kind = state[kCrossStatusWord] >= 1 && state[kCrossStatusWord] <= 6 ? state[kCrossStatusWord] : 0;
            CUDA_CHECK(cudaMemset(state_.get<int>() + kCrossStatusWord, 0, sizeof(int)));
            settle_legacy_stream();
            throw CudaFailure(std::string("the cross key/value projection gave up waiting for ") + kinds[kind], false);
        }
        if (state[kError] != 0) {
            CUDA_CHECK(cudaMemset(state_.get<int>() + kError, 0, sizeof(int)));
            settle_legacy_stream();
            if (state[kError] & kErrBarrierTimeout) {
                static const char* const kinds[] = {"?", "a grid barrier", "a weight unit", "a free stage",
                                                    "a landing copy", "an armed stage", "the splits of a product"};
                const int kind = state[kFailKind] >= 1 && state[kFailKind] <= 6 ? state[kFailKind] : 0;
                CUDA_CHECK(cudaMemset(state_.get<int>() + kFailKind, 0, 3 * sizeof(int)));
                settle_legacy_stream();
                throw CudaFailure(std::string("the decode kernel gave up waiting for ") + kinds[kind] + " (CTA " +
                                      std::to_string(state[kFailCta]) + ", index " +
                                      std::to_string(state[kFailWhere]) + ")",
                                  false);
            }
            throw ModelError("a sampled or supplied token id fell outside the vocabulary");
        }
    }

    static int op_class(int kind) {
        switch (kind) {
        case kOpEmbed: return WSP_KERNEL_EMBED;
        case kOpProduct: return WSP_KERNEL_PROJECTION;
        case kOpSelfAttention: return WSP_KERNEL_SELF_ATTENTION;
        case kOpCrossAttention: return WSP_KERNEL_CROSS_ATTENTION;
        case kOpLogits: return WSP_KERNEL_LOGITS_ARGMAX;
        case kOpNorm: return WSP_KERNEL_LAYER_NORM;
        }
        return WSP_KERNEL_OTHER;
    }

    // Keys a CTA-wide attention item scores at once beyond the self
    // capacity (the self attention holds max_positions scores).
    static constexpr int kMaxCrossChunk = 0;
    static constexpr int kMaxBlocksPerSm = 2;
    static constexpr int kStaticSharedBytes = 2048;
    static constexpr int kMinStages = 3;
    static constexpr int kFfnParts = 4;  // K parts of a few-row fc2

    // The step: recordDecoderStep (Decoder.cpp:151-177) with decoderLayer
    // (Decoder.cpp:73-115), lowered onto the ops of step.cuh.
    // With more rows than this, each LayerNorm runs once as a norm op rather
    // than in the prologue of every CTA's product.
    static constexpr int kInlineNormRows = 8;

    // A product's LayerNorm prologue (gamma, beta), or -- past
    // kInlineNormRows rows -- a norm op ahead of it and the product reading
    // the normalised rows.
    void normalised_input(std::vector<StepOp>& ops, StepOp& product, const DeviceBuffer& gamma,
                          const DeviceBuffer& beta, int R) const {
        if (R <= kInlineNormRows) {
            product.gamma = gamma.get<float>();
            product.beta = beta.get<float>();
            return;
        }
        StepOp norm{};
        norm.kind = kOpNorm;
        norm.gamma = gamma.get<float>();
        norm.beta = beta.get<float>();
        norm.out = normalised_.get();
        norm.ld_out = padded(shape_.width);
        norm.norm_rows = R;
        norm.norm_step = 1;
        norm.norm_offset = 0;
        norm.norm_umma = umma_ ? 1 : 0;
        ops.push_back(norm);
        product.input16 = normalised_.get();
        product.ld_input = padded(shape_.width);
    }

    std::vector<StepOp> build_ops(int R, int grid, int stage_bytes, const StepParams& p) const {
        const int d = shape_.width, f = shape_.feed_forward_width, H = shape_.heads;
        const int kpd = padded(d), kpf = padded(f);
        const size_t elem = 2;
        const size_t self_layer = (size_t)windows_ * shape_.max_positions * d * elem;
        const CrossSplit cs = cross_split(R, grid, stage_bytes);
        // A few rows, 64-wide heads, mma.sync products, every (row, head) on a
        // CTA of its own: each attention op applies its heads' out-projection
        // shares itself, and the LayerNorm prologue of the op after it adds
        // them to h (in head order, with the bias); the cross attention
        // computes its own queries -- three grid-wide phases fewer per layer.
        // h holds a layer's input and output rows, hidden_mid_ the rows
        // between its self and cross attention.
        const bool fuse_out = !umma_ && R <= kInlineNormRows && d == 64 * H && (long long)R * H < grid;
        float* self_partials = out_partials_.get<float>();
        float* cross_partials = self_partials + (size_t)H * std::min(R, kInlineNormRows) * d;
        // With the out-projections fused, fc2 (a few tiles of a long K) also
        // splits its K over kFfnParts items a tile, each writing its sums
        // apart; the next layer's LayerNorm prologue adds the parts and the
        // bias to h, keeping the new residual rows in hidden_alt_ (which the
        // cross attention then reads), so no CTA reads rows another rewrites
        // in the same op.  The last layer's fc2 adds to h itself: the logits
        // read h.
        const int ffn_tiles = (d + 15) / 16 * ((R + 7) / 8);
        const bool split_ffn = fuse_out && kpf != kpd && (kpf / 32) % kFfnParts == 0 &&
                               (long long)ffn_tiles * kFfnParts <= grid;
        float* ffn_partials = ffn_partials_.get<float>();
        std::vector<StepOp> ops;
        StepOp e{};
        e.kind = kOpEmbed;
        ops.push_back(e);
        for (int l = 0; l < shape_.layers; ++l) {
            const LayerBuffers& W = layers_[l];
            auto product = [&](int epilogue, const DeviceBuffer& w, int n, int kp, const DeviceBuffer& bias) {
                StepOp o{};
                o.kind = kOpProduct;
                o.epilogue = epilogue;
                o.weight = w.get();
                o.n = n;
                o.kp = kp;
                o.bias = bias.get<float>();
                return o;
            };
            // h += out_proj(self_attention(self_attn_layer_norm(h)))  (Decoder.cpp:80-91)
            const int D = d / H;
            StepOp qkv = product(kEpQkv, W.qkv_w, H * (int)round16(3 * D), kpd, W.qkv_b);
            normalised_input(ops, qkv, W.ln1_w, W.ln1_b, R);
            qkv.out = queries_.get();
            qkv.ld_out = d;
            qkv.self_keys = self_keys_.get<char>() + l * self_layer;
            qkv.self_values = self_values_.get<char>() + l * self_layer;
            qkv.prefetch_keys = fuse_out ? 1 : 0;
            if (split_ffn && l > 0) {
                // The previous layer's fc2 parts and bias, added to h.
                qkv.addends = ffn_partials;
                qkv.addend_count = kFfnParts;
                qkv.addend_stride = (long long)R * d;
                qkv.addend_bias = layers_[l - 1].fc2_b.get<float>();
                qkv.sum_out = hidden_alt_.get<float>();
            }
            ops.push_back(qkv);
            StepOp self{};
            self.kind = kOpSelfAttention;
            self.keys = qkv.self_keys;
            self.values = qkv.self_values;
            self.key_stride = d;
            self.window_stride = (long long)shape_.max_positions * d;
            if (fuse_out) {
                self.out_weight = W.o_w.get();
                self.out_partial = self_partials;
            }
            ops.push_back(self);
            if (!fuse_out) {
                StepOp out = product(kEpResidual, W.o_w, d, kpd, W.o_b);
                out.input16 = attended_.get();
                out.ld_input = kpd;
                out.out = hidden_.get();
                out.ld_out = d;
                ops.push_back(out);
            }
            // h += out_proj(cross_attention(encoder_attn_layer_norm(h)))  (Decoder.cpp:93-104)
            StepOp cross{};
            if (fuse_out) {
                // The cross attention computes its own queries: LN2 of h plus
                // the self attention's partials (the residual, kept in
                // hidden_mid_), then the head's q rows of W_q.
                cross = product(kEpStore, W.qc_w, H * (int)round16(D), kpd, W.qc_b);
                cross.gamma = W.ln2_w.get<float>();
                cross.beta = W.ln2_b.get<float>();
                cross.addends = self_partials;
                cross.addend_count = H;
                cross.addend_stride = (long long)R * d;
                cross.addend_bias = W.o_b.get<float>();
                cross.sum_out = hidden_mid_.get<float>();
                if (split_ffn && l > 0) cross.norm_input = hidden_alt_.get<float>();
            } else {
                StepOp cq = product(kEpStore, W.qc_w, H * (int)round16(D), kpd, W.qc_b);
                cq.slice = D;
                normalised_input(ops, cq, W.ln2_w, W.ln2_b, R);
                cq.out = queries_.get();
                cq.ld_out = d;
                ops.push_back(cq);
            }
            cross.kind = kOpCrossAttention;
            const long long head_block = (long long)shape_.cross_positions * 2 * D;
            // [layer][window][head][X][K | V]: the layer's blocks for every window together.
            cross.keys = cross_kv_.get<char>() + (size_t)l * windows_ * H * head_block * elem;
            cross.key_stride = 2 * D;
            cross.head_stride = head_block;
            cross.window_stride = (long long)H * head_block;
            cross.key_count = active_cross_;
            cross.chunk = cs.chunk;
            cross.span = cs.span;
            cross.splits = cs.splits;
            cross.value_bias = W.vc_b.get<float>();
            if (fuse_out) {
                cross.out_weight = W.oc_w.get();
                cross.out_partial = cross_partials;
            }
            ops.push_back(cross);
            if (!fuse_out) {
                StepOp cout = product(kEpResidual, W.oc_w, d, kpd, W.oc_b);
                cout.input16 = attended_.get();
                cout.ld_input = kpd;
                cout.out = hidden_.get();
                cout.ld_out = d;
                ops.push_back(cout);
            }
            // h += fc2(gelu(fc1(final_layer_norm(h))))  (Decoder.cpp:106-114)
            StepOp up = product(kEpGelu, W.fc1_w, f, kpd, W.fc1_b);
            normalised_input(ops, up, W.ln3_w, W.ln3_b, R);
            if (fuse_out) {
                up.norm_input = hidden_mid_.get<float>();
                up.addends = cross_partials;
                up.addend_count = H;
                up.addend_stride = (long long)R * d;
                up.addend_bias = W.oc_b.get<float>();
                up.sum_out = hidden_.get<float>();
            }
            up.out = feed_forward_.get();
            up.ld_out = kpf;
            ops.push_back(up);
            StepOp down = product(kEpResidual, W.fc2_w, d, kpf, W.fc2_b);
            down.input16 = feed_forward_.get();
            down.ld_input = kpf;
            down.out = hidden_.get();
            down.ld_out = d;
            if (split_ffn && l + 1 < shape_.layers) {
                down.epilogue = kEpPartial;
                down.kparts = kFfnParts;
                down.out = ffn_partials;
            }
            ops.push_back(down);
        }
        // Final layer norm and the tied logits with the masked argmax
        // (Decoder.cpp:170-176, Whisper::encodeSampling Whisper.cpp:1169-1184).
        StepOp logits{};
        logits.kind = kOpLogits;
        if (p.out_rows > kInlineNormRows) {
            StepOp norm{};
            norm.kind = kOpNorm;
            norm.gamma = final_w_.get<float>();
            norm.beta = final_b_.get<float>();
            norm.out = normalised_.get();
            norm.ld_out = kpd;
            norm.norm_rows = p.out_rows;
            norm.norm_step = p.row_step;
            norm.norm_offset = p.row_offset;
            norm.norm_hidden = p.hidden_out;
            norm.norm_umma = umma_ ? 1 : 0;  // the tcgen05 logits read the block layout
            ops.push_back(norm);
            logits.input16 = normalised_.get();
            logits.ld_input = kpd;
        }
        ops.push_back(logits);
        return ops;
    }

    // How a step splits its cross attention: `chunk` keys per stream unit (a
    // stage's worth), and for each (row, head) `splits` items of `span`
    // units.  A CTA works through its items one after another, so the cost
    // is its items' units plus a fixed cost per item (the query load, and
    // with several splits the join), in units.
    struct CrossSplit { int chunk, span, splits; };
    CrossSplit cross_split(int R, int grid, int stage_bytes) const {
        const int D = head_width();
        int chunk = std::max(1, std::min({kMaxCrossUnitKeys, stage_bytes / (4 * D), active_cross_}));
        // 64-wide heads run 16-key groups, dealt to the kStepWarps warps: a
        // unit takes as long as its busiest warp, so take the multiple of 16
        // that best trades the warps' balance against the stage it fills.
        if (D == 64 && chunk >= 16) {
            int best = chunk;
            double best_score = -1.0;
            for (int c = chunk / 16 * 16; c >= 16; c -= 16) {
                const int groups = c / 16, rounds = (groups + kStepWarps - 1) / kStepWarps;
                const double score = (double)groups / (kStepWarps * rounds) * c / chunk;
                if (score > best_score + 1e-9) {
                    best_score = score;
                    best = c;
                }
            }
            chunk = best;
        }
        // Units start on a multiple of 8 keys: the period of the rotated layout.
        if (chunk < active_cross_) chunk = std::max(8, chunk / 8 * 8);
        const int units = (active_cross_ + chunk - 1) / chunk;
        const long long pairs = (long long)R * shape_.heads;
        CrossSplit best{chunk, units, 1};
        double best_cost = 1e30;
        for (int span = 1; span <= units; ++span) {
            const int splits = (units + span - 1) / span;
            if (splits > kMaxCrossSplits) continue;
            const long long per_cta = (pairs * splits + grid - 1) / grid;
            const double cost = (double)per_cta * (span + (splits > 1 ? 2.0 : 1.0));
            if (cost < best_cost) {
                best_cost = cost;
                best = CrossSplit{chunk, span, splits};
            }
        }
        return best;
    }

    // Tensor-core products: a product whose (128-row weight tile, row
    // group) items fill less than half the grid splits its inner size so
    // that its items still fit one wave -- each split on its own CTA, which
    // lets the tile's splits meet and join their partials.  Returns the
    // partials' size in bytes.
    size_t split_products(std::vector<StepOp>& ops, const StepParams& p, int grid) const {
        size_t partial_bytes = 0;
        const int groups = (p.rows + p.umma_rows - 1) / p.umma_rows;
        for (StepOp& op : ops) {
            if (op.kind != kOpProduct || !p.umma) continue;
            const int m_tiles = (op.n + 127) / 128, kblocks = op.kp / 64;
            const int base = m_tiles * groups;
            int ks = 2 * base > grid ? 1 : std::min(kblocks, grid / base);
            if (ks > 1) {
                const int per = (kblocks + ks - 1) / ks;
                ks = (kblocks + per - 1) / per;
            }
            op.ksplit = ks;
            if (ks > 1) partial_bytes = std::max(partial_bytes, (size_t)ks * m_tiles * 128 * groups * p.umma_rows * 4);
        }
        return partial_bytes;
    }

    // Single-token steps of the tensor-core path: a split q/k/v product's
    // join moves into the self attention after it (StepOp::defer_join), which
    // sums its (row, head)'s partials in split order -- the same sums the
    // join would make -- so the product ends at its partials, without a
    // meeting of its splits.  Only where the self attention runs a warp per
    // (row, head) over 64-wide heads, and with one token a row, so no item
    // reads a key another item of the op writes.
    void defer_qkv_joins(std::vector<StepOp>& ops, const StepParams& p, int grid) const {
        if (!p.umma || p.tokens != 1 || p.head_width != 64 || p.max_positions > kSelfWarpKeys ||
            (long long)p.rows * p.heads < grid)
            return;
        const int groups = (p.rows + p.umma_rows - 1) / p.umma_rows;
        for (size_t i = 0; i + 1 < ops.size(); ++i) {
            StepOp& qkv = ops[i];
            StepOp& self = ops[i + 1];
            if (qkv.kind != kOpProduct || qkv.epilogue != kEpQkv || qkv.ksplit <= 1 ||
                self.kind != kOpSelfAttention || self.out_weight)
                continue;
            const int m_tiles = (qkv.n + 127) / 128, row_stride = groups * p.umma_rows;
            qkv.defer_join = 1;
            self.qkv_partial = p.partial_d;
            self.qkv_split_stride = (long long)m_tiles * row_stride * 128;
            self.qkv_row_stride = row_stride;
            self.qkv_splits = qkv.ksplit;
            self.qkv_bias = qkv.bias;
        }
    }

    // The tensor-core path: a split residual product (the out-projections,
    // fc2) followed by a norm op over every row leaves its join to that norm
    // (StepOp::defer_join): the norm's CTA for a row sums the row's partials
    // in split order, adds the bias and then the residual row -- the sums the
    // join and its atomic add would make -- writes the new residual row back
    // to h and normalises it.  The product ends at its partials, without a
    // meeting of its splits.
    void defer_residual_joins(std::vector<StepOp>& ops, const StepParams& p) const {
        if (!p.umma) return;
        const int groups = (p.rows + p.umma_rows - 1) / p.umma_rows, row_stride = groups * p.umma_rows;
        for (size_t i = 0; i + 1 < ops.size(); ++i) {
            StepOp& product = ops[i];
            StepOp& norm = ops[i + 1];
            if (product.kind != kOpProduct || product.epilogue != kEpResidual || product.ksplit <= 1 ||
                product.defer_join || !product.bias || product.out != static_cast<void*>(p.h) ||
                product.ld_out != p.width || norm.kind != kOpNorm || !norm.norm_umma || norm.addend_count > 0 ||
                norm.norm_rows != p.rows || norm.norm_step != 1 || norm.norm_offset != 0)
                continue;
            const int m_tiles = (product.n + 127) / 128;
            product.defer_join = 1;
            norm.addends = p.partial_d;
            norm.addend_count = product.ksplit;
            norm.addend_stride = (long long)m_tiles * row_stride * 128;
            norm.addend_tile_rows = row_stride;
            norm.addend_bias = product.bias;
            norm.sum_out = p.h;
        }
    }

    // The weight-stream schedule of every CTA (schedule.h), into device memory.
    void upload_schedule(StepParams& p, const std::vector<StepOp>& ops, int grid) {
        build_schedule(p, ops, grid, decode_tile_rows(p), schedule_host_, offsets_host_);
        if (schedule_host_.empty()) schedule_host_.push_back(ScheduleEntry{0, 0});
        const size_t entry = sizeof(ScheduleEntry);
        if (schedule_dev_.bytes() < schedule_host_.size() * entry)
            schedule_dev_.allocate(schedule_host_.size() * entry * 2);
        if (offsets_dev_.bytes() < offsets_host_.size() * 4) offsets_dev_.allocate(offsets_host_.size() * 4 * 2);
        check_schedule(p.stage_bytes);
        CUDA_CHECK(cudaMemcpyAsync(schedule_dev_.get(), schedule_host_.data(), schedule_host_.size() * entry,
                                   cudaMemcpyHostToDevice, stream_));
        CUDA_CHECK(cudaMemcpyAsync(offsets_dev_.get(), offsets_host_.data(), offsets_host_.size() * 4,
                                   cudaMemcpyHostToDevice, stream_));
        p.schedule = schedule_dev_.get<ScheduleEntry>();
        p.schedule_offsets = offsets_dev_.get<unsigned>();
    }

    // Every unit must lie inside one weight allocation, start 16-byte aligned
    // and fit a stage: checked on the host before any launch, so a bad
    // schedule is an error here rather than a fault on the device.
    void check_schedule(int stage_bytes) const {
        std::vector<std::pair<size_t, size_t>> ranges;
        auto add = [&](const DeviceBuffer& b) {
            if (b.get()) ranges.push_back({(size_t)b.get(), (size_t)b.get() + b.bytes()});
        };
        add(token_table_);
        add(cross_kv_);
        add(normalised_);
        add(attended_);
        add(feed_forward_);
        for (int l = 0; l < shape_.layers; ++l) {
            const LayerBuffers& W = layers_[l];
            add(W.qkv_w); add(W.o_w); add(W.qc_w); add(W.oc_w); add(W.fc1_w); add(W.fc2_w);
        }
        std::sort(ranges.begin(), ranges.end());
        for (size_t i = 0; i < schedule_host_.size(); ++i) {
            const ScheduleEntry& e = schedule_host_[i];
            if (e.source == 0 && e.bytes == 0) continue;  // the placeholder of an empty schedule
            if (e.bytes & kPrefetchOnly) continue;          // an L2 prefetch, not a unit
            const size_t bytes = (size_t)e.bytes;
            const size_t lo = (size_t)e.source, hi = lo + bytes;
            auto it = std::upper_bound(ranges.begin(), ranges.end(), std::make_pair(lo, (size_t)-1));
            const bool inside = it != ranges.begin() && lo >= std::prev(it)->first && hi <= std::prev(it)->second;
            if (!inside || lo % 16 != 0 || bytes % 16 != 0 || bytes == 0 || bytes > (size_t)stage_bytes)
                throw LogicError("weight-stream unit " + std::to_string(i) + " lies outside the weights");
        }
    }

    // Stage size: one 16-row tile over kpd (at least 16 KB); as many stages
    // (2..kMaxStreamStages) as the shared memory left by the work area holds.
    int stage_bytes_for_width() const {
        const int tile = 16 * padded(shape_.width) * 2;
        return std::max(16384, (tile + 1023) / 1024 * 1024);
    }

    // The weight stream's stages: as many as the shared memory left by the
    // work area holds.  Should a tile of 32 input rows (its hi and lo planes)
    // leave fewer than kMinStages, the tiles shrink to 16 rows, then 8.
    void configure_stream(bool half, StepParams& p) const {
        p.stage_bytes = stage_bytes_for_width();
        for (int columns = 4; columns >= 1; columns /= 2) {
            p.tile_columns = columns;
            const size_t work = decode_work_bytes(half, p, kMaxCrossChunk);
            // (The kernel's static shared memory -- barriers, flags, a fused
            // out-projection's input row -- comes out of the same budget.)
            const long long room = (long long)max_shared_ - kStaticSharedBytes - (long long)work;
            p.stages = (int)std::min<long long>(kMaxStreamStages, room / p.stage_bytes);
            if (p.stages >= kMinStages) return;
        }
        if (p.stages < 2) throw CudaFailure("the decode kernel's shared memory does not fit", false);
    }

    StepParams base_params(int T, bool sample, const float* mask, float* logits, float* hidden,
                           uint32_t* row_tokens, int steps, bool stop) const {
        const int R = windows_ * T;
        StepParams p{};
        p.windows = windows_;
        p.tokens = T;
        p.rows = R;
        p.width = shape_.width;
        p.heads = shape_.heads;
        p.head_width = shape_.width / shape_.heads;
        p.ffn = shape_.feed_forward_width;
        p.vocabulary = shape_.vocabulary_size;
        p.kpd = padded(shape_.width);
        p.umma = umma_ ? 1 : 0;
        p.act_rows = act_rows();
        p.max_positions = shape_.max_positions;
        p.ring_stride = ring_stride();
        p.scale = 1.f / std::sqrt((float)p.head_width);
        p.out_rows = sample ? windows_ : R;
        p.row_step = sample ? T : 1;
        p.row_offset = sample ? T - 1 : 0;
        p.ring = ring_.get<uint32_t>();
        p.state = state_.get<int>();
        p.token_table = token_table_.get();
        p.position_table = position_table_.get<float>();
        p.final_gamma = final_w_.get<float>();
        p.final_beta = final_b_.get<float>();
        p.h = hidden_.get<float>();
        p.q = queries_.get<float>();
        p.attn16 = attended_.get();
        p.ffn16 = feed_forward_.get();
        p.partial = partial_.get<float>();
        p.combine_counters = counters_.get<unsigned>();
        p.logits_counter = counters_.get<unsigned>() + (size_t)windows_ * token_capacity_ * shape_.heads;
        p.candidate_values = candidate_values_.get<float>();
        p.candidate_indices = candidate_indices_.get<uint32_t>();
        p.barrier = barrier_.get<unsigned>();
        p.mask = mask;
        p.logits_out = logits;
        p.hidden_out = hidden;
        p.row_tokens = row_tokens;
        p.ended = ended_.get<uint8_t>();
        p.write_ring = sample ? 1 : 0;
        p.steps = steps;
        p.stop_token = end_of_text_;
        p.stop_enabled = stop ? 1 : 0;

        return p;
    }

    // One launch of the decode kernel: `steps` steps of T tokens per window.
    // sample: only each window's last row is normalised, projected and
    // sampled into the ring; otherwise every row's logits/hidden/argmax.
    const std::vector<StepOp>& launch_steps(int T, bool sample, const float* mask, float* logits, float* hidden,
                                            uint32_t* row_tokens, int steps, bool stop,
                                            unsigned long long* profile) {
        const int R = windows_ * T;
        StepParams p = base_params(T, sample, mask, logits, hidden, row_tokens, steps, stop);
        p.profile = profile;
        const bool half = storage_ == Storage::f16;
        // A tensor-core item's rows: as many as a weight stage holds (128
        // bytes a row), at most 128, a multiple of 16; the activation ring
        // holds three k-blocks of that many rows, each its hi plane then its
        // lo plane (two products into one accumulator).  (Two stages of 128
        // rows, leaving a fourth weight stage, measured 14 % slower in the
        // large-v3 cross attention at 128 windows.)
        p.stage_bytes = stage_bytes_for_width();
        p.umma_rows = std::min(128, p.stage_bytes / 128 / 16 * 16);
        if (umma_) {
            p.umma_x_stage_bytes = 2 * std::min(p.umma_rows, (R + 15) / 16 * 16) * 128;
            p.umma_x_stages = 3;
            p.umma_blocks = std::max(1, p.stage_bytes / 16384);
        }
        configure_stream(half, p);
        const int blocks = decode_blocks_per_sm(half, p, kMaxCrossChunk);
        if (blocks <= 0) throw CudaFailure("the decode kernel does not fit on an SM", false);
        const int grid = sm_count_ * std::min(blocks, kMaxBlocksPerSm);
        std::vector<StepOp>& ops = sample ? (T == 1 ? ops_step_ : ops_prompt_) : ops_teacher_;
        DeviceBuffer& ops_dev = sample ? (T == 1 ? ops_step_dev_ : ops_prompt_dev_) : ops_teacher_dev_;
        ops = build_ops(R, grid, p.stage_bytes, p);
        const size_t partial_bytes = split_products(ops, p, grid);
        if (partial_d_.bytes() < partial_bytes) partial_d_.allocate(partial_bytes);
        p.partial_d = partial_d_.get<float>();
        defer_qkv_joins(ops, p, grid);
        defer_residual_joins(ops, p);
        if (umma_) {
            const size_t counter_bytes = ops.size() * kSplitSlots * sizeof(unsigned);
            if (split_counters_.bytes() < counter_bytes) split_counters_.allocate(counter_bytes);
            CUDA_CHECK(cudaMemsetAsync(split_counters_.get(), 0, counter_bytes, stream_));
            p.split_counters = split_counters_.get<unsigned>();
        }
        if (ops_dev.bytes() < ops.size() * sizeof(StepOp)) ops_dev.allocate(ops.size() * sizeof(StepOp));
        CUDA_CHECK(cudaMemcpyAsync(ops_dev.get(), ops.data(), ops.size() * sizeof(StepOp), cudaMemcpyHostToDevice,
                                   stream_));
        p.ops = ops_dev.get<StepOp>();
        p.n_ops = (int)ops.size();
        upload_schedule(p, ops, grid);
        // The abort and steps-done words; the all-ended flag survives from
        // the prompt step to the steps after it.
        CUDA_CHECK(cudaMemsetAsync(state_.get<int>() + kAbort, 0, 2 * sizeof(int), stream_));
        CUDA_CHECK(cudaMemsetAsync(barrier_.get(), 0, barrier_.bytes(), stream_));
        // The cross attention's (row, head) counters: a launch whose splits
        // join together counts them up from zero.
        CUDA_CHECK(cudaMemsetAsync(counters_.get(), 0,
                                   (size_t)windows_ * token_capacity_ * shape_.heads * sizeof(unsigned), stream_));
        try {
            launch_decode(half, p, kMaxCrossChunk, grid, stream_);
        } catch (const std::runtime_error& e) {
            throw CudaFailure(e.what(), false);
        }
        ++launches_;
        return ops;
    }

    // ------------------------------------------------------ upload helpers

    // The narrowing of a projection matrix (or the token table) to the
    // storage type.  WSP_NARROW_EXACT is the reference's ExactHalf rule
    // (Model/SafeTensors.h:146-159, DecoderWeights.cpp:149-178): narrow only
    // a tensor every value of which survives unchanged.  Where the reference
    // then keeps the fp32 tensor, this decoder (16-bit weights only) refuses
    // it, naming the tensor and the first value that would change.  The
    // default, WSP_NARROW_ROUND, rounds to nearest even; either way the
    // tensors narrowed inexactly and the largest change are counted.
    void audit_narrowing(const std::string& name, wsp_dtype dtype, const void* data, size_t count) {
        if (dtype != WSP_FLOAT32 && ((dtype == WSP_FLOAT16) == (storage_ == Storage::f16))) return;  // same type
        double largest = 0.0;
        size_t first = count;
        for (size_t i = 0; i < count; ++i) {
            const float v = widen(data, dtype, i);
            const float back = widen16(narrow(v, storage_));
            if (!(back == v) && !(std::isnan(v) && std::isnan(back))) {
                if (first == count) first = i;
                largest = std::max(largest, (double)std::fabs(back - v));
            }
        }
        if (first == count) return;
        if (narrowing_ == WSP_NARROW_EXACT)
            throw ModelError(name + " does not narrow exactly to " +
                             (storage_ == Storage::f16 ? "float16" : "bfloat16") + ": element " +
                             std::to_string(first) + " is " + std::to_string(widen(data, dtype, first)));
        ++inexact_tensors_;
        largest_change_ = std::max(largest_change_, largest);
    }

    float widen16(uint16_t bits) const {
        return widen(&bits, storage_ == Storage::f16 ? WSP_FLOAT16 : WSP_BFLOAT16, 0);
    }

public:
    void set_narrowing(int mode) {
        if (mode != WSP_NARROW_ROUND && mode != WSP_NARROW_EXACT)
            throw InvalidArgument("narrowing must be WSP_NARROW_ROUND or WSP_NARROW_EXACT");
        narrowing_ = mode;
    }
    void narrowing_stats(int* tensors, double* largest) const {
        if (tensors) *tensors = inexact_tensors_;
        if (largest) *largest = largest_change_;
    }

private:

    static std::string describe(const int64_t* extents, int rank) {
        std::string s = "[";
        for (int i = 0; i < rank; ++i) s += (i ? ", " : "") + std::to_string(extents[i]);
        return s + "]";
    }

    static void require_extents(const std::string& name, const int64_t* extents, int rank,
                                std::initializer_list<int> expected) {
        bool ok = rank == (int)expected.size();
        int i = 0;
        for (int e : expected) {
            if (ok && extents[i] != e) ok = false;
            ++i;
        }
        if (!ok) {
            std::string want = "[";
            i = 0;
            for (int e : expected) want += (i++ ? ", " : "") + std::to_string(e);
            throw ModelError(name + " has shape " + describe(extents, rank) + ", expected " + want + "]");
        }
    }

    // Narrows a [rows, cols] tensor into a 16-bit buffer at the element
    // offsets map(r, c) gives, keeping the buffer's other elements.
    template <typename Map>
    void patch16(DeviceBuffer& dst, int rows, int cols, wsp_dtype dtype, const void* data, Map map) {
        std::vector<uint16_t> v(dst.bytes() / 2);
        CUDA_CHECK(cudaMemcpy(v.data(), dst.get(), v.size() * 2, cudaMemcpyDeviceToHost));
        for (int r = 0; r < rows; ++r)
            for (int c = 0; c < cols; ++c)
                v[map(r, c)] = narrow(widen(data, dtype, (size_t)r * cols + c), storage_);
        CUDA_CHECK(cudaMemcpy(dst.get(), v.data(), v.size() * 2, cudaMemcpyHostToDevice));
    }

    template <typename Map>
    void patch_floats(DeviceBuffer& dst, int count, wsp_dtype dtype, const void* data, Map map) {
        std::vector<float> v(dst.bytes() / 4);
        CUDA_CHECK(cudaMemcpy(v.data(), dst.get(), v.size() * 4, cudaMemcpyDeviceToHost));
        for (int i = 0; i < count; ++i) v[map(i)] = widen(data, dtype, (size_t)i);
        CUDA_CHECK(cudaMemcpy(dst.get(), v.data(), v.size() * 4, cudaMemcpyHostToDevice));
    }

    // q_proj (0), k_proj (1) or v_proj (2) into the head-grouped q/k/v matrix.
    void patch_qkv(DeviceBuffer& dst, int which, wsp_dtype dtype, const void* data) {
        const int d = shape_.width, chunks = padded(d) / 32;
        (void)chunks;
        patch16(dst, d, d, dtype, data, [&](int r, int c) { return weight_offset(qkv_row(which, r), c, padded(d)); });
    }

    void upload_floats(DeviceBuffer& dst, size_t offset, size_t count, wsp_dtype dtype, const void* data) {
        std::vector<float> v(count);
        for (size_t i = 0; i < count; ++i) v[i] = widen(data, dtype, i);
        CUDA_CHECK(cudaMemcpy(dst.get<float>() + offset, v.data(), count * 4, cudaMemcpyHostToDevice));
    }

    // Cross k_proj (kv 0) or v_proj (kv 1) of a layer into the projection
    // that writes the cross caches: per layer and head, the head's D key rows
    // then its D value rows -- weight row ((layer * H + head) * 2 + kv) * D +
    // i -- so the product of a window's encoder rows with one (layer, head)
    // group's 2D rows is [X][K | V]; stored in the tensor-core layout
    // (cross_weight_offset) in the host copy.
    void upload_cross_projection(int layer, int kv, wsp_dtype dtype, const void* data) {
        const int d = shape_.width, H = shape_.heads, D = d / H, kblocks = (d + kCrossBlockCols - 1) / kCrossBlockCols;
        for (int h = 0; h < H; ++h)
            for (int i = 0; i < D; ++i) {
                const int n = ((layer * H + h) * 2 + kv) * D + i;
                const size_t src = (size_t)(h * D + i) * d;
                for (int c = 0; c < d; ++c)
                    cross_kv_host_[cross_weight_offset(n, c, kblocks)] = narrow(widen(data, dtype, src + c), storage_);
            }
        cross_weights_dirty_ = true;
    }

    // Elements of the cross projection's weights: L*2d rows in whole tiles,
    // d columns in whole k-blocks (cross_weight_offset).
    size_t cross_weight_elements() const {
        const size_t rows = (size_t)2 * shape_.width * shape_.layers;
        const size_t tiles = (rows + kCrossTileRows - 1) / kCrossTileRows;
        const size_t kblocks = (shape_.width + kCrossBlockCols - 1) / kCrossBlockCols;
        return tiles * kblocks * kCrossTileRows * kCrossBlockCols;
    }

    // rows x cols of a row-major [rows, cols] tensor into rows
    // [row_offset, row_offset+rows) of a fragment-packed [*, kp] matrix
    // (packed_offset, step.cuh), narrowed to the storage type.  The tiles
    // touched are read back first, since a tile may hold rows of two tensors.
    void upload_packed(DeviceBuffer& dst, int row_offset, int rows, int cols, int kp, wsp_dtype dtype,
                       const void* data) {
        const int chunks = kp / 32;
        const int t0 = row_offset / 16, t1 = (row_offset + rows - 1) / 16;
        const size_t tile_elements = (size_t)16 * kp;
        std::vector<uint16_t> v((size_t)(t1 - t0 + 1) * tile_elements);
        uint16_t* base = dst.get<uint16_t>() + (size_t)t0 * tile_elements;
        CUDA_CHECK(cudaMemcpy(v.data(), base, v.size() * 2, cudaMemcpyDeviceToHost));
        for (int r = 0; r < rows; ++r)
            for (int c = 0; c < cols; ++c)
                v[packed_offset(row_offset + r, c, chunks) - (size_t)t0 * tile_elements] =
                    narrow(widen(data, dtype, (size_t)r * cols + c), storage_);
        CUDA_CHECK(cudaMemcpy(base, v.data(), v.size() * 2, cudaMemcpyHostToDevice));
    }

    static void copy_floats(float* out, const float* in, size_t n) {
        if (is_device_pointer(in)) CUDA_CHECK(cudaMemcpy(out, in, n * 4, cudaMemcpyDeviceToHost));
        else std::memcpy(out, in, n * 4);
    }

    wsp_decoder_shape shape_;
    int device_;
    int windows_;
    Storage storage_;
    int sm_count_ = 148;
    int max_shared_ = 232448;
    cudaStream_t stream_ = nullptr;
    cudaEvent_t phase_events_[4] = {nullptr, nullptr, nullptr, nullptr};

    DeviceBuffer token_table_, position_table_, final_w_, final_b_, cross_kv_w_;
    std::unique_ptr<LayerBuffers[]> layers_;
    std::vector<bool> present_;

    DeviceBuffer self_keys_, self_values_, cross_kv_, encoder_staging_;
    // The cross projection's weights in their tensor-core layout, kept on the
    // host too so each k_proj / v_proj upload patches it; copied to the
    // device once before the next sequence start.
    std::vector<uint16_t> cross_kv_host_;
    bool cross_weights_dirty_ = false;
    DeviceBuffer ring_, ring_prompt_, state_, masks_;
    DeviceBuffer hidden_, queries_, normalised_, attended_, feed_forward_, partial_, partial_d_, split_counters_;
    DeviceBuffer out_partials_, hidden_mid_, hidden_alt_, ffn_partials_;
    DeviceBuffer candidate_values_, candidate_indices_, row_tokens_, counters_;
    DeviceBuffer barrier_, ended_, profile_;
    DeviceBuffer logits_staging_, hidden_staging_;
    DeviceBuffer ops_prompt_dev_, ops_step_dev_, ops_teacher_dev_, ops_probe_dev_;
    DeviceBuffer schedule_dev_, offsets_dev_;
    std::vector<ScheduleEntry> schedule_host_;
    std::vector<unsigned> offsets_host_;
    std::vector<StepOp> ops_prompt_, ops_step_, ops_teacher_;

    int token_capacity_ = 0;
    bool umma_ = false;
    int active_cross_ = 0;
    int position_ = 0;
    bool started_ = false;
    long long launches_ = 0;

    std::vector<uint32_t> prompt_;
    int maximum_tokens_ = 0;
    uint32_t end_of_text_ = 0;
    bool stop_at_end_of_text_ = true;
    bool generation_set_ = false;
    int sampled_steps_ = 0;
    std::vector<double> trace_cycles_;
    std::vector<double> op_us_;
    std::vector<int> op_kinds_;
    static constexpr int kTraceOffset = 512;   // kTraceBase of step.cu
    // The state word (after the decode kernel's) the cross projection
    // reports a wait that gave up in.
    static constexpr int kCrossStatusWord = kStateWords;
    static constexpr int kTraceSections = 16;
    int queued_steps_ = 0;
    int narrowing_ = WSP_NARROW_ROUND;
    int inexact_tensors_ = 0;
    double largest_change_ = 0.0;
};

}  // namespace
}  // namespace wsp

struct wsp_decoder {
    std::unique_ptr<wsp::Decoder> impl;
};

using wsp::guarded;

extern "C" {

const char* wsp_last_error(void) { return wsp::last_error_text().c_str(); }

int wsp_abi_version(void) { return WSP_ABI_VERSION; }

int wsp_device_count(int* count) {
    return guarded([&] {
        if (!count) throw wsp::InvalidArgument("count is NULL");
        wsp::cuda_check(cudaGetDeviceCount(count), "cudaGetDeviceCount");
    });
}

int wsp_decoder_create_products(const wsp_decoder_shape* shape, int device, int windows, wsp_dtype storage,
                                int products, wsp_decoder** out) {
    return guarded([&] {
        if (!shape || !out) throw wsp::InvalidArgument("shape and out must not be NULL");
        *out = nullptr;
        if (storage != WSP_FLOAT16 && storage != WSP_BFLOAT16)
            throw wsp::InvalidArgument("storage must be WSP_FLOAT16 or WSP_BFLOAT16");
        if (products != WSP_PRODUCTS_AUTO && products != WSP_PRODUCTS_MMA && products != WSP_PRODUCTS_TCGEN05)
            throw wsp::InvalidArgument("products must be WSP_PRODUCTS_AUTO, WSP_PRODUCTS_MMA or WSP_PRODUCTS_TCGEN05");
        auto holder = std::make_unique<wsp_decoder>();
        holder->impl = std::make_unique<wsp::Decoder>(
            *shape, device, windows, storage == WSP_FLOAT16 ? wsp::Storage::f16 : wsp::Storage::bf16, products);
        *out = holder.release();
    });
}

int wsp_decoder_create(const wsp_decoder_shape* shape, int device, int windows, wsp_dtype storage,
                       wsp_decoder** out) {
    return wsp_decoder_create_products(shape, device, windows, storage, WSP_PRODUCTS_AUTO, out);
}

void wsp_decoder_destroy(wsp_decoder* decoder) { delete decoder; }

#define WSP_NEED(decoder) \
    if (!(decoder) || !(decoder)->impl) throw wsp::InvalidArgument("decoder is NULL")

int wsp_decoder_set_tensor(wsp_decoder* decoder, const char* name, wsp_dtype dtype, const int64_t* extents,
                           int rank, const void* data) {
    return guarded([&] {
        WSP_NEED(decoder);
        decoder->impl->set_tensor(name, dtype, extents, rank, data);
        wsp::settle_legacy_stream();  // the uploads are pageable copies
    });
}

int wsp_decoder_set_narrowing(wsp_decoder* decoder, int mode) {
    return guarded([&] {
        WSP_NEED(decoder);
        decoder->impl->set_narrowing(mode);
    });
}

int wsp_decoder_narrowing(const wsp_decoder* decoder, int* inexact_tensors, double* largest_change) {
    return guarded([&] {
        WSP_NEED(decoder);
        decoder->impl->narrowing_stats(inexact_tensors, largest_change);
    });
}

int wsp_decoder_check_weights(const wsp_decoder* decoder) {
    return guarded([&] {
        WSP_NEED(decoder);
        decoder->impl->check_weights();
    });
}

int wsp_decoder_begin_sequence(wsp_decoder* decoder, const float* encoder_rows, int cross_positions) {
    return guarded([&] {
        WSP_NEED(decoder);
        decoder->impl->begin_sequence(encoder_rows, cross_positions);
    });
}

int wsp_decoder_step(wsp_decoder* decoder, const uint32_t* tokens, int token_count, float* logits, float* hidden,
                     uint32_t* argmax) {
    return guarded([&] {
        WSP_NEED(decoder);
        decoder->impl->step(tokens, token_count, logits, hidden, argmax);
    });
}

int wsp_decoder_position(const wsp_decoder* decoder, int* position) {
    return guarded([&] {
        WSP_NEED(decoder);
        if (!position) throw wsp::InvalidArgument("position is NULL");
        *position = decoder->impl->position();
    });
}

int wsp_decoder_cross_positions(const wsp_decoder* decoder, int* cross_positions) {
    return guarded([&] {
        WSP_NEED(decoder);
        if (!cross_positions) throw wsp::InvalidArgument("cross_positions is NULL");
        *cross_positions = decoder->impl->cross_positions();
    });
}

int wsp_decoder_set_generation(wsp_decoder* decoder, const wsp_generation_config* config) {
    return guarded([&] {
        WSP_NEED(decoder);
        if (!config) throw wsp::InvalidArgument("config is NULL");
        decoder->impl->set_generation(*config);
    });
}

int wsp_decoder_transcribe(wsp_decoder* decoder, const float* encoder_rows, int cross_positions, uint32_t* tokens,
                           int32_t* counts) {
    return guarded([&] {
        WSP_NEED(decoder);
        decoder->impl->transcribe(encoder_rows, cross_positions, tokens, counts);
    });
}

int wsp_decoder_enqueue_transcribe(wsp_decoder* decoder, const float* encoder_rows, int cross_positions,
                                   int steps) {
    return guarded([&] {
        WSP_NEED(decoder);
        decoder->impl->enqueue_transcribe(encoder_rows, cross_positions, steps);
    });
}

int wsp_decoder_read_transcript(wsp_decoder* decoder, uint32_t* tokens, int32_t* counts) {
    return guarded([&] {
        WSP_NEED(decoder);
        decoder->impl->read_transcript(tokens, counts);
    });
}

void* wsp_decoder_stream(wsp_decoder* decoder) {
    return decoder && decoder->impl ? (void*)decoder->impl->stream() : nullptr;
}

int wsp_decoder_synchronize(wsp_decoder* decoder) {
    return guarded([&] {
        WSP_NEED(decoder);
        decoder->impl->synchronize();
    });
}

int wsp_decoder_time_kernels(wsp_decoder* decoder, int steps, float* ms, int* launches) {
    return guarded([&] {
        WSP_NEED(decoder);
        decoder->impl->time_kernels(steps, ms, launches);
    });
}

int wsp_decoder_time_barriers(wsp_decoder* decoder, int count, float* microseconds) {
    return guarded([&] {
        WSP_NEED(decoder);
        if (!microseconds) throw wsp::InvalidArgument("microseconds is NULL");
        *microseconds = decoder->impl->time_barriers(count);
    });
}

int wsp_decoder_trace_cycles(const wsp_decoder* decoder, double* cycles, int count) {
    return guarded([&] {
        WSP_NEED(decoder);
        if (!cycles || count < 0) throw wsp::InvalidArgument("cycles is NULL");
        decoder->impl->trace_cycles(cycles, count);
    });
}

int wsp_decoder_op_times(const wsp_decoder* decoder, float* microseconds, int* kinds, int capacity, int* count) {
    return guarded([&] {
        WSP_NEED(decoder);
        if (capacity < 0 || !count) throw wsp::InvalidArgument("count is NULL or capacity negative");
        *count = decoder->impl->op_times(microseconds, kinds, capacity);
    });
}

int wsp_decoder_phase_ms(wsp_decoder* decoder, float* ms) {
    return guarded([&] {
        WSP_NEED(decoder);
        if (!ms) throw wsp::InvalidArgument("ms is NULL");
        decoder->impl->phase_ms(ms);
    });
}

int wsp_decoder_step_launches(const wsp_decoder* decoder, int* launches) {
    return guarded([&] {
        WSP_NEED(decoder);
        if (!launches) throw wsp::InvalidArgument("launches is NULL");
        *launches = decoder->impl->step_launches();
    });
}

int wsp_argmax(const float* logits, const float* mask, uint32_t* indices, int row_count, int row_length,
               void* stream) {
    return guarded([&] {
        if (!logits || !indices) throw wsp::InvalidArgument("logits and indices must not be NULL");
        if (row_count <= 0 || row_length <= 0) throw wsp::InvalidArgument("argmax needs rows of positive length");
        cudaStream_t s = static_cast<cudaStream_t>(stream);
        const int groups = wsp::argmax_groups_per_row(row_length);
        float* cv = nullptr;
        uint32_t* ci = nullptr;
        wsp::cuda_check(cudaMallocAsync(&cv, (size_t)row_count * groups * 4, s), "cudaMallocAsync");
        wsp::cuda_check(cudaMallocAsync(&ci, (size_t)row_count * groups * 4, s), "cudaMallocAsync");
        wsp::launch_argmax_rows(logits, mask, indices, row_count, row_length, cv, ci, groups, s);
        wsp::cuda_check(cudaGetLastError(), "argmax launch");
        cudaFreeAsync(cv, s);
        cudaFreeAsync(ci, s);
        wsp::cuda_check(cudaStreamSynchronize(s), "argmax");
    });
}

int wsp_argmax_no_alloc(const float* logits, const float* mask, uint32_t* indices, int row_count,
                        int row_length, void* stream) {
    return guarded([&] {
        if (!logits || !indices) throw wsp::InvalidArgument("logits and indices must not be NULL");
        if (row_count <= 0 || row_length <= 0) throw wsp::InvalidArgument("argmax needs rows of positive length");
        const int groups = wsp::argmax_groups_per_row(row_length);
        if ((long long)row_count * groups > wsp::kNoAllocArgmaxCandidates)
            throw wsp::InvalidArgument("wsp_argmax_no_alloc holds at most " +
                                       std::to_string(wsp::kNoAllocArgmaxCandidates) +
                                       " row groups (rows x ceil(length / 2048)); " + std::to_string(row_count) +
                                       " rows of " + std::to_string(row_length) + " need " +
                                       std::to_string((long long)row_count * groups));
        int device = 0;
        wsp::cuda_check(cudaGetDevice(&device), "cudaGetDevice");
        void* scratch = nullptr;
        wsp::cuda_check(wsp::no_alloc_argmax_scratch(device, &scratch), "cudaGetSymbolAddress (argmax scratch)");
        float* values = static_cast<float*>(scratch);
        uint32_t* candidates = reinterpret_cast<uint32_t*>(values + wsp::kNoAllocArgmaxCandidates);
        wsp::launch_argmax_rows(logits, mask, indices, row_count, row_length, values, candidates, groups,
                                static_cast<cudaStream_t>(stream));
        wsp::cuda_check(cudaGetLastError(), "argmax launch");
    });
}

}  // extern "C"
