// Host side of the B200 decoder: weights, caches, the step recording, the
// greedy search loop, and the C ABI of include/wsp_decoder.h.
//
// Reference (paths within eyalamirmusic/WhisperEACP):
//   Decoder / recordDecoderStep / recordSequenceStart  Lib/WhisperEACP/Decoder/Decoder.{h,cpp}
//   DecoderWeights                                     Lib/WhisperEACP/Decoder/DecoderWeights.{h,cpp}
//   greedy search                                      Lib/WhisperEACP/Whisper/Whisper.cpp:148-254,1158-1449
#include "../../include/wsp_decoder.h"
#include "kernels.cuh"

#include <cublas_v2.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

namespace wsp {
namespace {

// -------------------------------------------------------------- errors

struct ModelError : std::runtime_error { using std::runtime_error::runtime_error; };
struct LogicError : std::logic_error { using std::logic_error::logic_error; };
struct InvalidArgument : std::invalid_argument { using std::invalid_argument::invalid_argument; };
struct CudaFailure : std::runtime_error {
    bool out_of_memory;
    CudaFailure(const std::string& what, bool oom) : std::runtime_error(what), out_of_memory(oom) {}
};

thread_local std::string last_error_text;

void cuda_check(cudaError_t e, const char* what) {
    if (e != cudaSuccess)
        throw CudaFailure(std::string(what) + ": " + cudaGetErrorString(e), e == cudaErrorMemoryAllocation);
}
#define CUDA_CHECK(x) cuda_check((x), #x)

void cublas_check(cublasStatus_t s, const char* what) {
    if (s != CUBLAS_STATUS_SUCCESS)
        throw CudaFailure(std::string(what) + ": cuBLAS status " + std::to_string((int)s),
                          s == CUBLAS_STATUS_ALLOC_FAILED);
}

// ------------------------------------------------------- device memory

class DeviceBuffer {
public:
    DeviceBuffer() = default;
    DeviceBuffer(const DeviceBuffer&) = delete;
    DeviceBuffer& operator=(const DeviceBuffer&) = delete;
    ~DeviceBuffer() { release(); }

    void allocate(size_t bytes) {
        release();
        if (bytes == 0) bytes = 16;
        CUDA_CHECK(cudaMalloc(&ptr_, bytes));
        CUDA_CHECK(cudaMemset(ptr_, 0, bytes));
        bytes_ = bytes;
    }
    void release() {
        if (ptr_) cudaFree(ptr_);
        ptr_ = nullptr;
        bytes_ = 0;
    }
    template <typename T = void> T* get() const { return static_cast<T*>(ptr_); }
    size_t bytes() const { return bytes_; }

private:
    void* ptr_ = nullptr;
    size_t bytes_ = 0;
};

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

// Per-kernel-class CUDA event timing for measurement runs.
struct KernelTimer {
    cudaStream_t stream;
    std::vector<std::pair<int, std::pair<cudaEvent_t, cudaEvent_t>>> marks;
    int open_class = -1;
    cudaEvent_t open_start = nullptr;

    cudaEvent_t make() {
        cudaEvent_t e;
        CUDA_CHECK(cudaEventCreate(&e));
        return e;
    }
    void begin(int cls) {
        open_class = cls;
        open_start = make();
        CUDA_CHECK(cudaEventRecord(open_start, stream));
    }
    void end() {
        cudaEvent_t stop = make();
        CUDA_CHECK(cudaEventRecord(stop, stream));
        marks.push_back({open_class, {open_start, stop}});
    }
    ~KernelTimer() {
        for (auto& m : marks) {
            cudaEventDestroy(m.second.first);
            cudaEventDestroy(m.second.second);
        }
    }
};

class Decoder {
public:
    Decoder(const wsp_decoder_shape& shape, int device, int windows, Storage storage)
        : shape_(shape), device_(device), windows_(windows), storage_(storage) {
        validate_shape();
        CUDA_CHECK(cudaSetDevice(device_));
        CUDA_CHECK(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking));
        CUDA_CHECK(cudaDeviceGetAttribute(&sm_count_, cudaDevAttrMultiProcessorCount, device_));
        cublas_check(cublasCreate(&cublas_), "cublasCreate");
        cublas_check(cublasSetStream(cublas_, stream_), "cublasSetStream");
        allocate_weights();
        allocate_state();
        ensure_row_capacity(4);
    }

    ~Decoder() {
        cudaSetDevice(device_);
        drop_graph();
        if (cublas_) cublasDestroy(cublas_);
        if (stream_) cudaStreamDestroy(stream_);
        if (pinned_ring_) cudaFreeHost(pinned_ring_);
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
                upload_matrix(token_table_, 0, shape_.vocabulary_size, d, padded(d), dtype, data);
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
        switch (which) {
        case 0: require_extents(name, extents, rank, {d}); upload_floats(L.ln1_w, 0, d, dtype, data); break;
        case 1: require_extents(name, extents, rank, {d}); upload_floats(L.ln1_b, 0, d, dtype, data); break;
        case 2: require_extents(name, extents, rank, {d, d}); upload_matrix(L.qkv_w, 0, d, d, kpd, dtype, data); break;
        case 3: require_extents(name, extents, rank, {d}); upload_floats(L.qkv_b, 0, d, dtype, data); break;
        case 4: require_extents(name, extents, rank, {d, d}); upload_matrix(L.qkv_w, d, d, d, kpd, dtype, data); break;
        case 5: require_extents(name, extents, rank, {d, d}); upload_matrix(L.qkv_w, 2 * d, d, d, kpd, dtype, data); break;
        case 6: require_extents(name, extents, rank, {d}); upload_floats(L.qkv_b, 2 * d, d, dtype, data); break;
        case 7: require_extents(name, extents, rank, {d, d}); upload_matrix(L.o_w, 0, d, d, kpd, dtype, data); break;
        case 8: require_extents(name, extents, rank, {d}); upload_floats(L.o_b, 0, d, dtype, data); break;
        case 9: require_extents(name, extents, rank, {d}); upload_floats(L.ln2_w, 0, d, dtype, data); break;
        case 10: require_extents(name, extents, rank, {d}); upload_floats(L.ln2_b, 0, d, dtype, data); break;
        case 11: require_extents(name, extents, rank, {d, d}); upload_matrix(L.qc_w, 0, d, d, kpd, dtype, data); break;
        case 12: require_extents(name, extents, rank, {d}); upload_floats(L.qc_b, 0, d, dtype, data); break;
        case 13:  // cross keys: rows [l*2d, l*2d+d) of the all-layer projection
            require_extents(name, extents, rank, {d, d});
            upload_matrix(cross_kv_w_, (size_t)layer * 2 * d, d, d, d, dtype, data);
            break;
        case 14:
            require_extents(name, extents, rank, {d, d});
            upload_matrix(cross_kv_w_, (size_t)layer * 2 * d + d, d, d, d, dtype, data);
            break;
        case 15: require_extents(name, extents, rank, {d}); upload_floats(L.vc_b, 0, d, dtype, data); break;
        case 16: require_extents(name, extents, rank, {d, d}); upload_matrix(L.oc_w, 0, d, d, kpd, dtype, data); break;
        case 17: require_extents(name, extents, rank, {d}); upload_floats(L.oc_b, 0, d, dtype, data); break;
        case 18: require_extents(name, extents, rank, {d}); upload_floats(L.ln3_w, 0, d, dtype, data); break;
        case 19: require_extents(name, extents, rank, {d}); upload_floats(L.ln3_b, 0, d, dtype, data); break;
        case 20: require_extents(name, extents, rank, {f, d}); upload_matrix(L.fc1_w, 0, f, d, kpd, dtype, data); break;
        case 21: require_extents(name, extents, rank, {f}); upload_floats(L.fc1_b, 0, f, dtype, data); break;
        case 22: require_extents(name, extents, rank, {d, f}); upload_matrix(L.fc2_w, 0, d, f, kpf, dtype, data); break;
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
        if (!is_device_pointer(encoder_rows)) {
            CUDA_CHECK(cudaMemcpyAsync(encoder_staging_.get(), encoder_rows, elements * sizeof(float),
                                       cudaMemcpyHostToDevice, stream_));
            source = encoder_staging_.get<float>();
        }
        launch_to_storage(storage_, source, encoder16_.get(), (long long)elements, stream_);
        ++launches_;

        // recordSequenceStart (Decoder.cpp:121-146): every layer's cross keys
        // and values in one product, [rows, 2dL] per window.  The value bias
        // is added after the attention instead (the weights sum to one).
        const int d = shape_.width, n = 2 * d * shape_.layers;
        const float one = 1.f, zero = 0.f;
        const cudaDataType_t type = storage_ == Storage::f16 ? CUDA_R_16F : CUDA_R_16BF;
        cublas_check(cublasGemmStridedBatchedEx(
                         cublas_, CUBLAS_OP_T, CUBLAS_OP_N, n, rows, d, &one, cross_kv_w_.get(), type, d, 0,
                         encoder16_.get(), type, d, (long long)shape_.cross_positions * d, &zero, cross_kv_.get(),
                         type, n, (long long)shape_.cross_positions * n, windows_, CUBLAS_COMPUTE_32F,
                         CUBLAS_GEMM_DEFAULT),
                     "cross key/value projection");
        CUDA_CHECK(cudaMemsetAsync(state_.get(), 0, 2 * sizeof(int), stream_));
        CUDA_CHECK(cudaGetLastError());
        if (rows != active_cross_) drop_graph();
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
        StepPlan plan;
        plan.tokens = count;
        plan.sample_last_only = false;
        plan.mask = nullptr;
        plan.logits = logits ? (logits_on_device ? logits : logits_staging_.get<float>()) : nullptr;
        plan.hidden = hidden ? (hidden_on_device ? hidden : hidden_staging_.get<float>()) : nullptr;
        plan.row_tokens = row_tokens_.get<uint32_t>();
        plan.write_ring = false;
        record_step(plan, nullptr);
        CUDA_CHECK(cudaGetLastError());
        if (logits && !logits_on_device)
            CUDA_CHECK(cudaMemcpyAsync(logits, plan.logits, (size_t)R * shape_.vocabulary_size * 4,
                                       cudaMemcpyDeviceToHost, stream_));
        if (hidden && !hidden_on_device)
            CUDA_CHECK(cudaMemcpyAsync(hidden, plan.hidden, (size_t)R * shape_.width * 4, cudaMemcpyDeviceToHost,
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
        begin_sequence(encoder_rows, cross_positions);
        CUDA_CHECK(cudaMemcpyAsync(ring_.get(), ring_prompt_.get(), ring_prompt_.bytes(), cudaMemcpyDeviceToDevice,
                                   stream_));
        StepPlan plan = sampling_plan((int)prompt_.size(), masks_.get<float>());
        record_step(plan, nullptr);
        CUDA_CHECK(cudaGetLastError());
        position_ = (int)prompt_.size();
        sampled_steps_ = 1;
    }

    // encodeStep for step k > 0 (Whisper.cpp:1207-1212), replayed as a graph.
    void enqueue_steps(int steps) {
        for (int i = 0; i < steps; ++i) {
            if (position_ + 1 > shape_.max_positions) throw ModelError("the window is full");
            launch_single_step_graph();
            ++position_;
            ++sampled_steps_;
        }
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
        const int steps = sampled_steps_;
        const int p = (int)prompt_.size();
        std::vector<uint32_t> ring((size_t)windows_ * ring_stride());
        CUDA_CHECK(cudaMemcpyAsync(ring.data(), ring_.get(), ring.size() * 4, cudaMemcpyDeviceToHost, stream_));
        CUDA_CHECK(cudaStreamSynchronize(stream_));
        check_device_errors();
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

    // Whisper::decodeTranscript (Whisper.cpp:1361-1449).  The host checks for
    // end-of-text every few steps rather than every step: the steps queued
    // past a window's end are computed and ignored, as the reference's
    // in-flight steps are.
    void transcribe(const float* encoder_rows, int cross_positions, uint32_t* tokens, int32_t* counts) {
        const int limit = step_limit();
        enqueue_start(encoder_rows, cross_positions);
        if (stop_at_end_of_text_) {
            if (!pinned_ring_) CUDA_CHECK(cudaMallocHost(&pinned_ring_, (size_t)windows_ * ring_stride() * 4));
            const int batch = 16;
            while (sampled_steps_ < limit) {
                const int n = std::min(batch, limit - sampled_steps_);
                enqueue_steps(n);
                CUDA_CHECK(cudaMemcpyAsync(pinned_ring_, ring_.get(), (size_t)windows_ * ring_stride() * 4,
                                           cudaMemcpyDeviceToHost, stream_));
                CUDA_CHECK(cudaStreamSynchronize(stream_));
                if (all_windows_ended(pinned_ring_)) break;
            }
        } else {
            enqueue_steps(limit - 1);
        }
        read_transcript(tokens, counts);
    }

    cudaStream_t stream() const { return stream_; }

    void synchronize() {
        CUDA_CHECK(cudaSetDevice(device_));
        CUDA_CHECK(cudaStreamSynchronize(stream_));
        check_device_errors();
    }

    // Launch-by-launch timing of single-token sampled steps.
    void time_kernels(int steps, float* ms, int* launches) {
        if (!generation_set_ || !started_) throw LogicError("time_kernels needs a transcription in progress");
        if (position_ + steps > shape_.max_positions) throw ModelError("not enough room left in the window");
        CUDA_CHECK(cudaSetDevice(device_));
        KernelTimer timer{stream_};
        for (int i = 0; i < steps; ++i) {
            StepPlan plan = sampling_plan(1, masks_.get<float>() + shape_.vocabulary_size);
            record_step(plan, &timer);
            ++position_;
        }
        CUDA_CHECK(cudaStreamSynchronize(stream_));
        std::vector<double> total(WSP_KERNEL_CLASSES, 0.0);
        std::vector<int> count(WSP_KERNEL_CLASSES, 0);
        for (auto& m : timer.marks) {
            float t = 0.f;
            CUDA_CHECK(cudaEventElapsedTime(&t, m.second.first, m.second.second));
            total[m.first] += t;
            count[m.first] += 1;
        }
        for (int c = 0; c < WSP_KERNEL_CLASSES; ++c) {
            if (ms) ms[c] = count[c] ? (float)(total[c] / count[c]) : 0.f;
            if (launches) launches[c] = steps ? count[c] / steps : 0;
        }
    }

    int step_launches() const { return 5 + 13 * shape_.layers; }

private:
    struct StepPlan {
        int tokens = 1;
        bool sample_last_only = true;
        const float* mask = nullptr;
        float* logits = nullptr;
        float* hidden = nullptr;
        uint32_t* row_tokens = nullptr;
        bool write_ring = true;
    };

    StepPlan sampling_plan(int tokens, const float* mask) {
        StepPlan plan;
        plan.tokens = tokens;
        plan.sample_last_only = true;
        plan.mask = mask;
        plan.write_ring = true;
        return plan;
    }

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

    void allocate_weights() {
        const size_t d = shape_.width, f = shape_.feed_forward_width, L = shape_.layers;
        const size_t kpd = padded(d), kpf = padded(f);
        token_table_.allocate((size_t)shape_.vocabulary_size * kpd * 2);
        position_table_.allocate((size_t)shape_.max_positions * d * 4);
        final_w_.allocate(d * 4);
        final_b_.allocate(d * 4);
        cross_kv_w_.allocate(2 * d * L * d * 2);
        layers_.reset(new LayerBuffers[L]);
        for (size_t i = 0; i < L; ++i) {
            LayerBuffers& l = layers_[i];
            l.ln1_w.allocate(d * 4); l.ln1_b.allocate(d * 4);
            l.qkv_w.allocate(3 * d * kpd * 2); l.qkv_b.allocate(3 * d * 4);
            l.o_w.allocate(d * kpd * 2); l.o_b.allocate(d * 4);
            l.ln2_w.allocate(d * 4); l.ln2_b.allocate(d * 4);
            l.qc_w.allocate(d * kpd * 2); l.qc_b.allocate(d * 4); l.vc_b.allocate(d * 4);
            l.oc_w.allocate(d * kpd * 2); l.oc_b.allocate(d * 4);
            l.ln3_w.allocate(d * 4); l.ln3_b.allocate(d * 4);
            l.fc1_w.allocate(f * kpd * 2); l.fc1_b.allocate(f * 4);
            l.fc2_w.allocate(d * kpf * 2); l.fc2_b.allocate(d * 4);
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
        encoder16_.allocate(B * X * d * 2);
        ring_.allocate(B * ring_stride() * 4);
        ring_prompt_.allocate(B * ring_stride() * 4);
        state_.allocate(2 * sizeof(int));
        masks_.allocate(2 * (size_t)shape_.vocabulary_size * 4);
        self_splits_ = (shape_.max_positions + kSelfChunk - 1) / kSelfChunk;
    }

    static constexpr int kSelfChunk = 64;

    int cross_splits(int cross_rows) const {
        const int pairs = windows_ * shape_.heads;
        int s = (2 * sm_count_ + pairs - 1) / pairs;
        s = std::max(s, (cross_rows + 2047) / 2048);
        s = std::min(s, std::max(1, (cross_rows + 31) / 32));
        return std::max(1, s);
    }

    void ensure_row_capacity(int tokens) {
        if (tokens <= token_capacity_) return;
        drop_graph();
        token_capacity_ = std::max(tokens, token_capacity_);
        const size_t R = (size_t)windows_ * token_capacity_;
        const size_t d = shape_.width, f = shape_.feed_forward_width, H = shape_.heads, D = d / H;
        const size_t splits = std::max(self_splits_, cross_splits(shape_.cross_positions));
        hidden_.allocate(R * d * 4);
        normalised_.allocate(R * padded(d) * 2);
        queries_.allocate(R * d * 4);
        attended_.allocate(R * padded(d) * 2);
        feed_forward_.allocate(R * padded(f) * 2);
        partial_.allocate(R * H * splits * (D + 2) * 4);
        const size_t tiles = gemm_column_tiles(shape_.vocabulary_size);
        candidate_values_.allocate(R * tiles * 4);
        candidate_indices_.allocate(R * tiles * 4);
        row_tokens_.allocate(R * 4);
        final_rows_hidden_.allocate(R * d * 4);
    }

    void ensure_staging(DeviceBuffer& buffer, size_t bytes) {
        if (buffer.bytes() < bytes) buffer.allocate(bytes);
    }

    void drop_graph() {
        if (graph_exec_) cudaGraphExecDestroy(graph_exec_);
        if (graph_) cudaGraphDestroy(graph_);
        graph_exec_ = nullptr;
        graph_ = nullptr;
    }

    void launch_single_step_graph() {
        if (!graph_exec_) {
            CUDA_CHECK(cudaStreamBeginCapture(stream_, cudaStreamCaptureModeThreadLocal));
            try {
                StepPlan plan = sampling_plan(1, masks_.get<float>() + shape_.vocabulary_size);
                record_step(plan, nullptr);
            } catch (...) {
                cudaGraph_t broken = nullptr;
                cudaStreamEndCapture(stream_, &broken);
                if (broken) cudaGraphDestroy(broken);
                throw;
            }
            CUDA_CHECK(cudaStreamEndCapture(stream_, &graph_));
            CUDA_CHECK(cudaGraphInstantiate(&graph_exec_, graph_, 0));
        }
        CUDA_CHECK(cudaGraphLaunch(graph_exec_, stream_));
    }

    bool all_windows_ended(const uint32_t* ring) const {
        const int p = (int)prompt_.size();
        for (int b = 0; b < windows_; ++b) {
            bool ended = false;
            for (int k = 0; k < sampled_steps_ && !ended; ++k)
                ended = ring[(size_t)b * ring_stride() + p + k] == end_of_text_;
            if (!ended) return false;
        }
        return true;
    }

    void check_device_errors() {
        int flags[2] = {0, 0};
        CUDA_CHECK(cudaMemcpy(flags, state_.get(), sizeof flags, cudaMemcpyDeviceToHost));
        if (flags[1] & 1) {
            CUDA_CHECK(cudaMemset(state_.get<int>() + 1, 0, sizeof(int)));
            throw ModelError("a sampled or supplied token id fell outside the vocabulary");
        }
    }

    // The step: recordDecoderStep (Decoder.cpp:151-177) with decoderLayer
    // (Decoder.cpp:73-115), lowered onto fused kernels.
    void record_step(const StepPlan& plan, KernelTimer* timer) {
        const int T = plan.tokens;
        const int R = windows_ * T;
        const int d = shape_.width, f = shape_.feed_forward_width, H = shape_.heads, D = d / H;
        const int kpd = padded(d), kpf = padded(f);
        const int L = shape_.layers;
        int* position = state_.get<int>();
        int* error = state_.get<int>() + 1;
        auto mark = [&](int cls) { if (timer) timer->begin(cls); };
        auto done = [&]() { ++launches_; if (timer) timer->end(); };

        EmbedArgs e{};
        e.ring = ring_.get<uint32_t>();
        e.ring_stride = ring_stride();
        e.position = position;
        e.tokens = T;
        e.rows = R;
        e.width = d;
        e.vocabulary = shape_.vocabulary_size;
        e.token_table = token_table_.get();
        e.token_stride = kpd;
        e.position_table = position_table_.get<float>();
        e.hidden = hidden_.get<float>();
        e.error = error;
        mark(WSP_KERNEL_EMBED);
        launch_embed(storage_, e, stream_);
        done();

        auto layer_norm = [&](const DeviceBuffer& w, const DeviceBuffer& b) {
            LayerNormArgs a{};
            a.input = hidden_.get<float>();
            a.rows = R;
            a.width = d;
            a.row_step = 1;
            a.row_offset = 0;
            a.gamma = w.get<float>();
            a.beta = b.get<float>();
            a.output = normalised_.get();
            a.ld_output = kpd;
            mark(WSP_KERNEL_LAYER_NORM);
            launch_layer_norm(storage_, a, stream_);
            done();
        };
        auto product = [&](Epilogue epi, const DeviceBuffer& w, int n, const void* input, int kp,
                           const float* bias, GemmArgs g) {
            g.weight = w.get();
            g.input = input;
            g.n = n;
            g.rows = R;
            g.kp = kp;
            g.bias = bias;
            mark(WSP_KERNEL_PROJECTION);
            launch_gemm(storage_, epi, g, sm_count_, stream_);
            done();
        };
        auto attend = [&](bool cross, int layer) {
            AttentionArgs a{};
            a.queries = queries_.get<float>();
            a.ld_queries = d;
            a.rows = R;
            a.tokens = T;
            a.heads = H;
            a.head_width = D;
            a.position = position;
            a.scale = 1.f / std::sqrt((float)D);
            a.partial = partial_.get<float>();
            const size_t bytes = storage_ == Storage::f16 ? 2 : 2;
            if (cross) {
                const size_t n = (size_t)2 * d * L;
                const char* base = cross_kv_.get<char>() + (size_t)layer * 2 * d * bytes;
                a.keys = base;
                a.values = base + (size_t)d * bytes;
                a.key_stride = (long long)n;
                a.window_stride = (long long)shape_.cross_positions * n;
                a.causal = 0;
                a.key_count = active_cross_;
                a.splits = cross_splits(active_cross_);
                a.chunk = (active_cross_ + a.splits - 1) / a.splits;
            } else {
                const size_t per_layer = (size_t)windows_ * shape_.max_positions * d * bytes;
                a.keys = self_keys_.get<char>() + layer * per_layer;
                a.values = self_values_.get<char>() + layer * per_layer;
                a.key_stride = d;
                a.window_stride = (long long)shape_.max_positions * d;
                a.causal = 1;
                a.splits = self_splits_;
                a.chunk = kSelfChunk;
            }
            mark(cross ? WSP_KERNEL_CROSS_ATTENTION : WSP_KERNEL_SELF_ATTENTION);
            launch_attention_partial(storage_, a, stream_);
            done();
            CombineArgs c{};
            c.partial = partial_.get<float>();
            c.rows = R;
            c.heads = H;
            c.head_width = D;
            c.splits = a.splits;
            c.bias = cross ? layers_[layer].vc_b.get<float>() : nullptr;
            c.output = attended_.get();
            c.ld_output = kpd;
            mark(WSP_KERNEL_ATTENTION_COMBINE);
            launch_attention_combine(storage_, c, stream_);
            done();
        };

        const size_t self_layer_elements = (size_t)windows_ * shape_.max_positions * d;
        for (int l = 0; l < L; ++l) {
            LayerBuffers& W = layers_[l];
            // h += out_proj(self_attention(self_attn_layer_norm(h)))  (Decoder.cpp:80-91)
            layer_norm(W.ln1_w, W.ln1_b);
            GemmArgs qkv{};
            qkv.out = queries_.get<float>();
            qkv.ld_out = d;
            qkv.width = d;
            qkv.self_keys = self_keys_.get<char>() + l * self_layer_elements * 2;
            qkv.self_values = self_values_.get<char>() + l * self_layer_elements * 2;
            qkv.max_positions = shape_.max_positions;
            qkv.tokens = T;
            qkv.position = position;
            product(Epilogue::qkv, W.qkv_w, 3 * d, normalised_.get(), kpd, W.qkv_b.get<float>(), qkv);
            attend(false, l);
            GemmArgs residual{};
            residual.out = hidden_.get<float>();
            residual.ld_out = d;
            product(Epilogue::residual, W.o_w, d, attended_.get(), kpd, W.o_b.get<float>(), residual);

            // h += out_proj(cross_attention(encoder_attn_layer_norm(h)))  (Decoder.cpp:93-104)
            layer_norm(W.ln2_w, W.ln2_b);
            GemmArgs q{};
            q.out = queries_.get<float>();
            q.ld_out = d;
            product(Epilogue::store, W.qc_w, d, normalised_.get(), kpd, W.qc_b.get<float>(), q);
            attend(true, l);
            product(Epilogue::residual, W.oc_w, d, attended_.get(), kpd, W.oc_b.get<float>(), residual);

            // h += fc2(gelu(fc1(final_layer_norm(h))))  (Decoder.cpp:106-114)
            layer_norm(W.ln3_w, W.ln3_b);
            GemmArgs up{};
            up.out16 = feed_forward_.get();
            up.ld_out16 = kpf;
            product(Epilogue::gelu, W.fc1_w, f, normalised_.get(), kpd, W.fc1_b.get<float>(), up);
            product(Epilogue::residual, W.fc2_w, d, feed_forward_.get(), kpf, W.fc2_b.get<float>(), residual);
        }

        // Final layer norm and the tied logits (Decoder.cpp:170-176); when
        // sampling, only each window's last row is normalised and projected
        // (Whisper::encodeSampling reads the last row, Whisper.cpp:1169-1184).
        const int out_rows = plan.sample_last_only ? windows_ : R;
        LayerNormArgs fl{};
        fl.input = hidden_.get<float>();
        fl.rows = out_rows;
        fl.width = d;
        fl.row_step = plan.sample_last_only ? T : 1;
        fl.row_offset = plan.sample_last_only ? T - 1 : 0;
        fl.gamma = final_w_.get<float>();
        fl.beta = final_b_.get<float>();
        fl.output = normalised_.get();
        fl.ld_output = kpd;
        fl.hidden_copy = plan.hidden;
        mark(WSP_KERNEL_LAYER_NORM);
        launch_layer_norm(storage_, fl, stream_);
        done();

        GemmArgs lg{};
        lg.weight = token_table_.get();
        lg.input = normalised_.get();
        lg.n = shape_.vocabulary_size;
        lg.rows = out_rows;
        lg.kp = kpd;
        lg.logits = plan.logits;
        lg.ld_logits = shape_.vocabulary_size;
        lg.mask = plan.mask;
        lg.candidate_values = candidate_values_.get<float>();
        lg.candidate_indices = candidate_indices_.get<uint32_t>();
        mark(WSP_KERNEL_LOGITS_ARGMAX);
        launch_gemm(storage_, Epilogue::logits, lg, sm_count_, stream_);
        done();

        ArgmaxFinalArgs af{};
        af.candidate_values = candidate_values_.get<float>();
        af.candidate_indices = candidate_indices_.get<uint32_t>();
        af.candidates = gemm_column_tiles(shape_.vocabulary_size);
        af.rows = out_rows;
        af.rows_per_window = plan.sample_last_only ? 1 : T;
        af.step_tokens = T;
        af.row_tokens = plan.row_tokens;
        af.ring = plan.write_ring ? ring_.get<uint32_t>() : nullptr;
        af.ring_stride = ring_stride();
        af.position = position;
        mark(WSP_KERNEL_ARGMAX_FINAL);
        launch_argmax_final(af, stream_);
        done();

        mark(WSP_KERNEL_OTHER);
        launch_advance_position(position, T, stream_);
        done();
    }

    // ------------------------------------------------------ upload helpers

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

    void upload_floats(DeviceBuffer& dst, size_t offset, size_t count, wsp_dtype dtype, const void* data) {
        std::vector<float> v(count);
        for (size_t i = 0; i < count; ++i) v[i] = widen(data, dtype, i);
        CUDA_CHECK(cudaMemcpy(dst.get<float>() + offset, v.data(), count * 4, cudaMemcpyHostToDevice));
    }

    // rows x cols of a row-major [rows, cols] tensor into dst rows
    // [row_offset, row_offset+rows) of pitch ld, narrowed to the storage type.
    void upload_matrix(DeviceBuffer& dst, size_t row_offset, int rows, int cols, int ld, wsp_dtype dtype,
                       const void* data) {
        std::vector<uint16_t> v((size_t)rows * ld, 0);
        for (int r = 0; r < rows; ++r)
            for (int c = 0; c < cols; ++c)
                v[(size_t)r * ld + c] = narrow(widen(data, dtype, (size_t)r * cols + c), storage_);
        CUDA_CHECK(cudaMemcpy(dst.get<uint16_t>() + row_offset * ld, v.data(), v.size() * 2, cudaMemcpyHostToDevice));
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
    cudaStream_t stream_ = nullptr;
    cublasHandle_t cublas_ = nullptr;

    DeviceBuffer token_table_, position_table_, final_w_, final_b_, cross_kv_w_;
    std::unique_ptr<LayerBuffers[]> layers_;
    std::vector<bool> present_;

    DeviceBuffer self_keys_, self_values_, cross_kv_, encoder_staging_, encoder16_;
    DeviceBuffer ring_, ring_prompt_, state_, masks_;
    DeviceBuffer hidden_, normalised_, queries_, attended_, feed_forward_, partial_;
    DeviceBuffer candidate_values_, candidate_indices_, row_tokens_, final_rows_hidden_;
    DeviceBuffer logits_staging_, hidden_staging_;
    uint32_t* pinned_ring_ = nullptr;

    int token_capacity_ = 0;
    int self_splits_ = 1;
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

    cudaGraph_t graph_ = nullptr;
    cudaGraphExec_t graph_exec_ = nullptr;
};

template <typename F>
int guarded(F&& f) {
    try {
        f();
        last_error_text.clear();
        return WSP_OK;
    } catch (const ModelError& e) {
        last_error_text = e.what();
        return WSP_MODEL_ERROR;
    } catch (const InvalidArgument& e) {
        last_error_text = e.what();
        return WSP_INVALID_ARGUMENT;
    } catch (const LogicError& e) {
        last_error_text = e.what();
        return WSP_LOGIC_ERROR;
    } catch (const CudaFailure& e) {
        last_error_text = e.what();
        return e.out_of_memory ? WSP_OUT_OF_MEMORY : WSP_CUDA_ERROR;
    } catch (const std::bad_alloc&) {
        last_error_text = "host allocation failed";
        return WSP_OUT_OF_MEMORY;
    } catch (const std::exception& e) {
        last_error_text = e.what();
        return WSP_LOGIC_ERROR;
    }
}

}  // namespace
}  // namespace wsp

struct wsp_decoder {
    std::unique_ptr<wsp::Decoder> impl;
};

using wsp::guarded;

extern "C" {

const char* wsp_last_error(void) { return wsp::last_error_text.c_str(); }

int wsp_abi_version(void) { return WSP_ABI_VERSION; }

int wsp_device_count(int* count) {
    return guarded([&] {
        if (!count) throw wsp::InvalidArgument("count is NULL");
        wsp::cuda_check(cudaGetDeviceCount(count), "cudaGetDeviceCount");
    });
}

int wsp_decoder_create(const wsp_decoder_shape* shape, int device, int windows, wsp_dtype storage,
                       wsp_decoder** out) {
    return guarded([&] {
        if (!shape || !out) throw wsp::InvalidArgument("shape and out must not be NULL");
        *out = nullptr;
        if (storage != WSP_FLOAT16 && storage != WSP_BFLOAT16)
            throw wsp::InvalidArgument("storage must be WSP_FLOAT16 or WSP_BFLOAT16");
        auto holder = std::make_unique<wsp_decoder>();
        holder->impl = std::make_unique<wsp::Decoder>(
            *shape, device, windows, storage == WSP_FLOAT16 ? wsp::Storage::f16 : wsp::Storage::bf16);
        *out = holder.release();
    });
}

void wsp_decoder_destroy(wsp_decoder* decoder) { delete decoder; }

#define WSP_NEED(decoder) \
    if (!(decoder) || !(decoder)->impl) throw wsp::InvalidArgument("decoder is NULL")

int wsp_decoder_set_tensor(wsp_decoder* decoder, const char* name, wsp_dtype dtype, const int64_t* extents,
                           int rank, const void* data) {
    return guarded([&] {
        WSP_NEED(decoder);
        decoder->impl->set_tensor(name, dtype, extents, rank, data);
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

}  // extern "C"
