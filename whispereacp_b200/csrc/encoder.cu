// The audio front end on B200: the log-mel spectrogram and the Whisper
// encoder (the C ABI of include/wsp_encoder.h).
//
// Reference (paths within eyalamirmusic/WhisperEACP):
//   MelSpectrogram   Lib/WhisperEACP/Mel/MelSpectrogram.cpp:101-196, MelKernels.h:43-255,
//                    Window.cpp (periodic Hann), Basis.cpp (the DFT basis)
//   Encoder          Lib/WhisperEACP/Encoder/Encoder.cpp:17-118 (recordEncoder, encoderLayer)
//   EncoderShape     Lib/WhisperEACP/Encoder/EncoderShape.cpp (positions, 1/sqrt(D) on the scores)
//
// Every product of the encoder -- the two convolutions (as products over
// their three taps), q/k/v, the out-projection, fc1 and fc2 -- runs on the
// tcgen05 tensor cores through the sequence start's product kernel
// (cross_kv.cuh) in its linear form: fp32 rows split into 16-bit hi + lo,
// 16-bit weights, an fp32 accumulator in tensor memory, and bias, GELU and
// the residual in the epilogue.  The spectrogram, the LayerNorms and the
// attention (1500 x 1500 a head) run on the CUDA cores in fp32.
#include "../../include/wsp_encoder.h"
#include "common.cuh"
#include "cross_kv.cuh"
#include "host.h"

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <memory>
#include <set>
#include <string>
#include <vector>

namespace wsp {
namespace {

constexpr int kFft = 400;                 // n_fft (Audio/Format.h)
constexpr int kHop = 160;                 // hop_length
constexpr int kBins = kFft / 2 + 1;       // 201
constexpr int kAttnTile = 64;             // queries and keys of an attention tile
constexpr int kHeadWidth = 64;
constexpr int kNormWarps = 8;

// ------------------------------------------------------------- spectrogram

// Frame f: the reflect-padded samples f*hop - n_fft/2 .. under the periodic
// Hann window (StftFramesKernel, MelKernels.h:43-70), then bin b's power
// re^2 + im^2 of its DFT against the basis (Basis.cpp), written [bin][frame]
// so the mel projection's reads are coalesced.
__global__ void __launch_bounds__(256) mel_power_kernel(const float* samples, int sample_count,
                                                        const float* window, const float* basis, float* power,
                                                        int frames) {
    __shared__ float x[kFft];
    const int f = blockIdx.x;
    const int last = sample_count - 1;
    for (int tap = threadIdx.x; tap < kFft; tap += blockDim.x) {
        const int index = f * kHop - kFft / 2 + tap;
        const int source = last - abs(last - abs(index));
        x[tap] = samples[source] * window[tap];
    }
    __syncthreads();
    const int b = threadIdx.x;
    if (b >= kBins) return;
    float re = 0.f, im = 0.f;
    for (int tap = 0; tap < kFft; ++tap) {
        const float2 w = *reinterpret_cast<const float2*>(basis + (size_t)tap * 2 * kBins + 2 * b);
        re += x[tap] * w.x;
        im += x[tap] * w.y;
    }
    power[(size_t)b * frames + f] = re * re + im * im;
}

// log10(max(filters . power, 1e-10)) (MelProjectKernel, MelKernels.h:120-150),
// [mel][frame].
__global__ void __launch_bounds__(128) mel_project_kernel(const float* power, const float* filters, float* log_mel,
                                                          int frames) {
    __shared__ float row[kBins];
    const int mel = blockIdx.y;
    for (int b = threadIdx.x; b < kBins; b += blockDim.x) row[b] = filters[(size_t)mel * kBins + b];
    __syncthreads();
    const int f = blockIdx.x * blockDim.x + threadIdx.x;
    if (f >= frames) return;
    float total = 0.f;
    for (int b = 0; b < kBins; ++b) total += row[b] * power[(size_t)b * frames + f];
    log_mel[(size_t)mel * frames + f] = log10f(fmaxf(total, 1e-10f));
}

// Per-block maxima of the log-mel (MaxReduceKernel, MelKernels.h:152-185).
__global__ void __launch_bounds__(256) max_partials_kernel(const float* values, int count, float* partials) {
    __shared__ float best[8];
    float m = -INFINITY;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < count; i += gridDim.x * blockDim.x) m = fmaxf(m, values[i]);
    m = warp_max(m);
    if ((threadIdx.x & 31) == 0) best[threadIdx.x >> 5] = m;
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < (int)(blockDim.x >> 5); ++w) m = fmaxf(m, best[w]);
        partials[blockIdx.x] = fmaxf(m, best[0]);
    }
}

// (max(x, peak - 8) + 4) / 4 (MelNormaliseKernel, MelKernels.h:187-210); each
// block folds the partial maxima itself.
__global__ void __launch_bounds__(256) mel_normalise_kernel(const float* values, int count, const float* partials,
                                                            int partial_count, float* out) {
    __shared__ float peak;
    if (threadIdx.x < 32) {
        float m = -INFINITY;
        for (int i = threadIdx.x; i < partial_count; i += 32) m = fmaxf(m, partials[i]);
        m = warp_max(m);
        if (threadIdx.x == 0) peak = m;
    }
    __syncthreads();
    const float floor_value = peak - 8.0f;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < count; i += gridDim.x * blockDim.x)
        out[i] = (fmaxf(values[i], floor_value) + 4.0f) / 4.0f;
}

// --------------------------------------------------------------- encoder

// The first convolution's product rows: row f holds, for channel c and tap
// t, mel[c][f + t - 1] (zero past either end): [frames][3 * mel_bins], the
// column order of the HF weight [width][mel_bins][3].
__global__ void conv1_columns_kernel(const float* mel, int mel_bins, int frames, float* columns) {
    const long long total = (long long)frames * 3 * mel_bins;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const int f = (int)(i / (3 * mel_bins)), j = (int)(i % (3 * mel_bins));
        const int c = j / 3, at = f + j % 3 - 1;
        columns[i] = at >= 0 && at < frames ? mel[(size_t)c * frames + at] : 0.f;
    }
}

// The second (stride 2): row p holds, for channel c and tap t, the first's
// output row 2p + t - 1: [positions][3 * width].
__global__ void conv2_columns_kernel(const float* first, int width, int frames, int positions, float* columns) {
    const long long total = (long long)positions * 3 * width;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const int p = (int)(i / (3 * width)), j = (int)(i % (3 * width));
        const int c = j / 3, at = 2 * p + j % 3 - 1;
        columns[i] = at >= 0 && at < frames ? first[(size_t)at * width + c] : 0.f;
    }
}

// LayerNorm (LayerNorm.h:19-98: the mean, then the centred variance, eps
// 1e-5) of `rows` rows of width d <= 32 * kNormPerLane, a warp a row.
constexpr int kNormPerLane = 48;
__global__ void __launch_bounds__(32 * kNormWarps) layer_norm_rows_kernel(const float* in, const float* gamma,
                                                                          const float* beta, float* out, int rows,
                                                                          int d) {
    const int row = blockIdx.x * kNormWarps + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (row >= rows) return;
    const float* x = in + (size_t)row * d;
    float v[kNormPerLane];
    float total = 0.f;
#pragma unroll
    for (int i = 0; i < kNormPerLane; ++i) {
        const int c = lane + 32 * i;
        v[i] = c < d ? x[c] : 0.f;
        total += v[i];
    }
    const float mean = warp_sum(total) / (float)d;
    float centred = 0.f;
#pragma unroll
    for (int i = 0; i < kNormPerLane; ++i) {
        const int c = lane + 32 * i;
        const float dv = c < d ? v[i] - mean : 0.f;
        centred += dv * dv;
    }
    const float scale = rsqrtf(warp_sum(centred) / (float)d + 1e-5f);
#pragma unroll
    for (int i = 0; i < kNormPerLane; ++i) {
        const int c = lane + 32 * i;
        if (c < d) out[(size_t)row * d + c] = (v[i] - mean) * scale * gamma[c] + beta[c];
    }
}

// Unmasked multi-head attention over `positions` rows (Net::attention with
// causal false; the reference's referenceAttention): qkv [positions][3d]
// (q, k, v side by side), out [positions][d].  A CTA takes 64 queries of one
// head and walks the keys 64 at a time with an online softmax in fp32; thread
// (ty, tx) holds queries 4ty..4ty+3 and keys (then output columns) tx +
// 16j.  Scores are scaled by 1/sqrt(D) (EncoderShape.cpp:38-44).
__global__ void __launch_bounds__(256) attention_kernel(const float* qkv, float* out, int positions, int d,
                                                        float scale) {
    extern __shared__ float smem[];
    constexpr int P = kAttnTile + 1;  // padded pitch
    float* qs = smem;                   // [64][65]
    float* ks = qs + kAttnTile * P;     // [64][65]
    float* vs = ks + kAttnTile * P;     // [64][64]
    float* ps = vs + kAttnTile * kAttnTile;  // [64][65]
    const int head = blockIdx.y, q0 = blockIdx.x * kAttnTile;
    const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;
    const size_t ld = (size_t)3 * d;
    for (int i = tid; i < kAttnTile * kHeadWidth; i += blockDim.x) {
        const int r = i / kHeadWidth, c = i % kHeadWidth;
        qs[r * P + c] = q0 + r < positions ? qkv[(size_t)(q0 + r) * ld + head * kHeadWidth + c] : 0.f;
    }
    float m[4], l[4], o[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        m[i] = -INFINITY;
        l[i] = 0.f;
#pragma unroll
        for (int j = 0; j < 4; ++j) o[i][j] = 0.f;
    }
    for (int k0 = 0; k0 < positions; k0 += kAttnTile) {
        __syncthreads();
        for (int i = tid; i < kAttnTile * kHeadWidth; i += blockDim.x) {
            const int r = i / kHeadWidth, c = i % kHeadWidth;
            const bool ok = k0 + r < positions;
            const float* row = qkv + (size_t)(k0 + r) * ld + head * kHeadWidth + c;
            ks[r * P + c] = ok ? row[d] : 0.f;
            vs[r * kAttnTile + c] = ok ? row[2 * d] : 0.f;
        }
        __syncthreads();
        float s[4][4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j) s[i][j] = 0.f;
        for (int c = 0; c < kHeadWidth; ++c) {
            float a[4], b[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) a[i] = qs[(4 * ty + i) * P + c];
#pragma unroll
            for (int j = 0; j < 4; ++j) b[j] = ks[(tx + 16 * j) * P + c];
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) s[i][j] += a[i] * b[j];
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            float rowmax = -INFINITY;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                s[i][j] = k0 + tx + 16 * j < positions ? scale * s[i][j] : -INFINITY;
                rowmax = fmaxf(rowmax, s[i][j]);
            }
#pragma unroll
            for (int x = 1; x < 16; x <<= 1) rowmax = fmaxf(rowmax, __shfl_xor_sync(0xffffffffu, rowmax, x));
            const float m_new = fmaxf(m[i], rowmax);
            const float keep = m[i] == -INFINITY ? 0.f : __expf(m[i] - m_new);
            float rowsum = 0.f;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float e = s[i][j] == -INFINITY ? 0.f : __expf(s[i][j] - m_new);
                ps[(4 * ty + i) * P + tx + 16 * j] = e;
                rowsum += e;
            }
#pragma unroll
            for (int x = 1; x < 16; x <<= 1) rowsum += __shfl_xor_sync(0xffffffffu, rowsum, x);
            l[i] = l[i] * keep + rowsum;
            m[i] = m_new;
#pragma unroll
            for (int j = 0; j < 4; ++j) o[i][j] *= keep;
        }
        __syncthreads();
        for (int c = 0; c < kAttnTile; ++c) {
            float a[4], b[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) a[i] = ps[(4 * ty + i) * P + c];
#pragma unroll
            for (int j = 0; j < 4; ++j) b[j] = vs[c * kAttnTile + tx + 16 * j];
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) o[i][j] += a[i] * b[j];
        }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int q = q0 + 4 * ty + i;
        if (q >= positions) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) out[(size_t)q * d + head * kHeadWidth + tx + 16 * j] = o[i][j] / l[i];
    }
}
constexpr size_t kAttentionSmem = sizeof(float) * (3 * kAttnTile * (kAttnTile + 1) + kAttnTile * kAttnTile);

// ------------------------------------------------------------------ host

enum class Storage { f16, bf16 };

float widen(const void* data, wsp_dtype dtype, size_t i) {
    switch (dtype) {
    case WSP_FLOAT32: return static_cast<const float*>(data)[i];
    case WSP_FLOAT16: return __half2float(*reinterpret_cast<const __half*>(static_cast<const uint16_t*>(data) + i));
    default: {
        const uint32_t bits = (uint32_t)static_cast<const uint16_t*>(data)[i] << 16;
        float f;
        std::memcpy(&f, &bits, 4);
        return f;
    }
    }
}

uint16_t narrow(float v, Storage s) {
    uint16_t bits;
    if (s == Storage::f16) {
        const __half h = __float2half_rn(v);
        std::memcpy(&bits, &h, 2);
    } else {
        const __nv_bfloat16 h = __float2bfloat16_rn(v);
        std::memcpy(&bits, &h, 2);
    }
    return bits;
}

// A product's weight: [n][k] in the tensor-core tile layout
// (cross_weight_offset), kept on the host until the first encode after a
// change.
struct Product {
    int n = 0, k = 0, kblocks = 0;
    std::vector<uint16_t> host;
    DeviceBuffer device;
    bool dirty = true;
    void shape(int rows, int cols) {
        n = rows;
        k = cols;
        kblocks = (k + kCrossBlockCols - 1) / kCrossBlockCols;
        host.assign((size_t)((n + kCrossTileRows - 1) / kCrossTileRows) * kCrossTileRows * kblocks * kCrossBlockCols,
                    0);
    }
    void put(int row0, int rows, const void* data, wsp_dtype dtype, Storage s) {
        for (int r = 0; r < rows; ++r)
            for (int c = 0; c < k; ++c)
                host[cross_weight_offset(row0 + r, c, kblocks)] = narrow(widen(data, dtype, (size_t)r * k + c), s);
        dirty = true;
    }
    void upload() {
        if (!dirty) return;
        if (device.bytes() < host.size() * 2) device.allocate(host.size() * 2);
        CUDA_CHECK(cudaMemcpy(device.get(), host.data(), host.size() * 2, cudaMemcpyHostToDevice));
        dirty = false;
    }
};

struct Vec {
    std::vector<float> host;
    DeviceBuffer device;
    bool dirty = true;
    void put(size_t offset, size_t count, const void* data, wsp_dtype dtype) {
        for (size_t i = 0; i < count; ++i) host[offset + i] = widen(data, dtype, i);
        dirty = true;
    }
    void upload() {
        if (!dirty) return;
        if (device.bytes() < host.size() * 4) device.allocate(host.size() * 4);
        CUDA_CHECK(cudaMemcpy(device.get(), host.data(), host.size() * 4, cudaMemcpyHostToDevice));
        dirty = false;
    }
    const float* get() const { return device.get<float>(); }
};

struct Layer {
    Vec ln1_w, ln1_b, qkv_b, o_b, ln2_w, ln2_b, fc1_b, fc2_b;
    Product qkv, o, fc1, fc2;
};

bool on_device(const void* p) {
    cudaPointerAttributes a{};
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged;
}

class Encoder {
public:
    Encoder(const wsp_encoder_shape& shape, int device, wsp_dtype storage) : shape_(shape), device_(device) {
        if (shape.mel_bins <= 0 || shape.width <= 0 || shape.heads <= 0 || shape.layers <= 0 ||
            shape.feed_forward_width <= 0 || shape.input_frames <= 1)
            throw ModelError("an encoder shape needs positive extents and at least two input frames");
        if (shape.width % shape.heads != 0 || shape.width / shape.heads != kHeadWidth)
            throw ModelError("this encoder needs 64-wide attention heads");
        if (shape.width > 32 * kNormPerLane || shape.width % 4 != 0 || shape.feed_forward_width % 4 != 0)
            throw ModelError("encoder width out of range");
        if (storage != WSP_FLOAT16 && storage != WSP_BFLOAT16)
            throw InvalidArgument("the encoder stores its weights as float16 or bfloat16");
        storage_ = storage == WSP_FLOAT16 ? Storage::f16 : Storage::bf16;
        int count = 0;
        CUDA_CHECK(cudaGetDeviceCount(&count));
        if (device < 0 || device >= count) throw InvalidArgument("no such CUDA device");
        CUDA_CHECK(cudaSetDevice(device));
        CUDA_CHECK(cudaDeviceGetAttribute(&sm_count_, cudaDevAttrMultiProcessorCount, device));
        CUDA_CHECK(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking));
        const int d = shape.width, f = shape.feed_forward_width, M = shape.mel_bins;
        positions_ = (shape.input_frames - 1) / 2 + 1;
        conv1_.shape(d, 3 * M);
        conv2_.shape(d, 3 * d);
        conv1_b_.host.assign(d, 0.f);
        conv2_b_.host.assign(d, 0.f);
        pos_.host.assign((size_t)positions_ * d, 0.f);
        final_w_.host.assign(d, 0.f);
        final_b_.host.assign(d, 0.f);
        filters_.host.assign((size_t)M * kBins, 0.f);
        for (int l = 0; l < shape.layers; ++l) layers_.push_back(std::make_unique<Layer>());
        for (auto& layer : layers_) {
            Layer& L = *layer;
            for (Vec* v : {&L.ln1_w, &L.ln1_b, &L.o_b, &L.ln2_w, &L.ln2_b, &L.fc2_b}) v->host.assign(d, 0.f);
            L.qkv_b.host.assign(3 * (size_t)d, 0.f);
            L.fc1_b.host.assign(f, 0.f);
            L.qkv.shape(3 * d, d);
            L.o.shape(d, d);
            L.fc1.shape(f, d);
            L.fc2.shape(d, f);
        }
        // The periodic Hann window (Window.cpp) and the DFT basis (Basis.cpp),
        // tap-major: [tap][cos of bin b at 2b, -sin at 2b + 1].
        window_.host.resize(kFft);
        for (int i = 0; i < kFft; ++i)
            window_.host[i] = (float)(0.5 * (1.0 - std::cos(2.0 * M_PI * (double)i / (double)kFft)));
        basis_.host.resize((size_t)kFft * 2 * kBins);
        for (int b = 0; b < kBins; ++b)
            for (int t = 0; t < kFft; ++t) {
                const double angle = 2.0 * M_PI * ((double)((b * t) % kFft) / (double)kFft);
                basis_.host[(size_t)t * 2 * kBins + 2 * b] = (float)std::cos(angle);
                basis_.host[(size_t)t * 2 * kBins + 2 * b + 1] = (float)-std::sin(angle);
            }
        const size_t F = shape.input_frames, P = positions_;
        samples_.allocate(F * kHop * 4);
        power_.allocate((size_t)kBins * F * 4);
        log_mel_.allocate((size_t)M * F * 4);
        mel_.allocate((size_t)M * F * 4);
        partials_.allocate(sm_count_ * 4);
        columns_.allocate(std::max((size_t)F * 3 * M, P * 3 * d) * 4);
        first_.allocate(F * d * 4);
        hidden_.allocate(P * d * 4);
        normed_.allocate(P * d * 4);
        qkv_.allocate(P * 3 * d * 4);
        attended_.allocate(P * d * 4);
        ffn_.allocate(P * f * 4);
        rows_.allocate(P * d * 4);
        status_.allocate(16);
        CUDA_CHECK(cudaFuncSetAttribute(attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        (int)kAttentionSmem));
    }
    ~Encoder() {
        cudaSetDevice(device_);
        if (stream_) cudaStreamDestroy(stream_);
    }

    // EncoderWeights (EncoderWeights.cpp): the HF names and extents.
    void set_tensor(const std::string& name, wsp_dtype dtype, const int64_t* extents, int rank, const void* data) {
        if (!data) throw InvalidArgument("tensor " + name + " has no data");
        if (dtype != WSP_FLOAT32 && dtype != WSP_FLOAT16 && dtype != WSP_BFLOAT16)
            throw InvalidArgument("tensor " + name + ": unknown element type");
        const int d = shape_.width, f = shape_.feed_forward_width, M = shape_.mel_bins;
        auto expect = [&](std::initializer_list<int64_t> want) {
            if (rank != (int)want.size() || !std::equal(want.begin(), want.end(), extents))
                throw ModelError("tensor " + name + " has the wrong shape");
        };
        const std::string prefix = "model.encoder.";
        if (name.rfind(prefix, 0) != 0) throw ModelError("tensor " + name + " is not an encoder tensor");
        const std::string rest = name.substr(prefix.size());
        if (rest == "conv1.weight") { expect({d, M, 3}); conv1_.put(0, d, data, dtype, storage_); }
        else if (rest == "conv1.bias") { expect({d}); conv1_b_.put(0, d, data, dtype); }
        else if (rest == "conv2.weight") { expect({d, d, 3}); conv2_.put(0, d, data, dtype, storage_); }
        else if (rest == "conv2.bias") { expect({d}); conv2_b_.put(0, d, data, dtype); }
        else if (rest == "embed_positions.weight") {
            if (rank != 2 || extents[1] != d || extents[0] < positions_)
                throw ModelError("tensor " + name + " has the wrong shape");
            pos_.put(0, (size_t)positions_ * d, data, dtype);
        }
        else if (rest == "layer_norm.weight") { expect({d}); final_w_.put(0, d, data, dtype); }
        else if (rest == "layer_norm.bias") { expect({d}); final_b_.put(0, d, data, dtype); }
        else if (rest.rfind("layers.", 0) == 0) {
            const size_t dot = rest.find('.', 7);
            const int l = std::atoi(rest.substr(7, dot - 7).c_str());
            if (dot == std::string::npos || l < 0 || l >= shape_.layers)
                throw ModelError("tensor " + name + " names no layer of this encoder");
            Layer& L = *layers_[l];
            const std::string t = rest.substr(dot + 1);
            if (t == "self_attn.q_proj.weight") { expect({d, d}); L.qkv.put(0, d, data, dtype, storage_); }
            else if (t == "self_attn.k_proj.weight") { expect({d, d}); L.qkv.put(d, d, data, dtype, storage_); }
            else if (t == "self_attn.v_proj.weight") { expect({d, d}); L.qkv.put(2 * d, d, data, dtype, storage_); }
            else if (t == "self_attn.q_proj.bias") { expect({d}); L.qkv_b.put(0, d, data, dtype); }
            else if (t == "self_attn.v_proj.bias") { expect({d}); L.qkv_b.put(2 * (size_t)d, d, data, dtype); }
            else if (t == "self_attn.out_proj.weight") { expect({d, d}); L.o.put(0, d, data, dtype, storage_); }
            else if (t == "self_attn.out_proj.bias") { expect({d}); L.o_b.put(0, d, data, dtype); }
            else if (t == "self_attn_layer_norm.weight") { expect({d}); L.ln1_w.put(0, d, data, dtype); }
            else if (t == "self_attn_layer_norm.bias") { expect({d}); L.ln1_b.put(0, d, data, dtype); }
            else if (t == "final_layer_norm.weight") { expect({d}); L.ln2_w.put(0, d, data, dtype); }
            else if (t == "final_layer_norm.bias") { expect({d}); L.ln2_b.put(0, d, data, dtype); }
            else if (t == "fc1.weight") { expect({f, d}); L.fc1.put(0, f, data, dtype, storage_); }
            else if (t == "fc1.bias") { expect({f}); L.fc1_b.put(0, f, data, dtype); }
            else if (t == "fc2.weight") { expect({d, f}); L.fc2.put(0, d, data, dtype, storage_); }
            else if (t == "fc2.bias") { expect({d}); L.fc2_b.put(0, d, data, dtype); }
            else throw ModelError("tensor " + name + " is not one this encoder reads");
        } else {
            throw ModelError("tensor " + name + " is not one this encoder reads");
        }
        seen_.insert(name);
    }

    void set_filters(const float* filters) {
        if (!filters) throw InvalidArgument("no filterbank");
        if (on_device(filters)) {
            CUDA_CHECK(cudaMemcpy(filters_.host.data(), filters, filters_.host.size() * 4, cudaMemcpyDeviceToHost));
        } else {
            std::memcpy(filters_.host.data(), filters, filters_.host.size() * 4);
        }
        filters_.dirty = true;
        filters_set_ = true;
    }

    void check_weights() const {
        for (const std::string& name : required_names())
            if (!seen_.count(name)) throw ModelError("the encoder has no tensor " + name);
    }

    void log_mel(const float* samples, int count, float* mel) {
        if (!samples || !mel) throw InvalidArgument("log_mel needs samples and an output");
        const int F = shape_.input_frames;
        if (count <= 1 || count > F * kHop)
            throw ModelError("a window holds 2 to " + std::to_string(F * kHop) + " samples, and this one has " +
                             std::to_string(count));
        if (!filters_set_) throw ModelError("the encoder has no mel filterbank");
        CUDA_CHECK(cudaSetDevice(device_));
        spectrogram(samples, count);
        copy_out(mel, mel_.get(), (size_t)shape_.mel_bins * F * 4);
    }

    void encode(const float* mel, float* rows) {
        if (!mel || !rows) throw InvalidArgument("encode needs a log-mel and an output");
        check_weights();
        CUDA_CHECK(cudaSetDevice(device_));
        const size_t bytes = (size_t)shape_.mel_bins * shape_.input_frames * 4;
        CUDA_CHECK(cudaMemcpyAsync(mel_.get(), mel, bytes, cudaMemcpyDefault, stream_));
        run_encoder();
        copy_out(rows, rows_.get(), (size_t)positions_ * shape_.width * 4);
    }

    void encode_samples(const float* samples, int count, float* rows) {
        if (!samples || !rows) throw InvalidArgument("encode needs samples and an output");
        check_weights();
        const int F = shape_.input_frames;
        if (count <= 1 || count > F * kHop)
            throw ModelError("a window holds 2 to " + std::to_string(F * kHop) + " samples, and this one has " +
                             std::to_string(count));
        if (!filters_set_) throw ModelError("the encoder has no mel filterbank");
        CUDA_CHECK(cudaSetDevice(device_));
        spectrogram(samples, count);
        run_encoder();
        copy_out(rows, rows_.get(), (size_t)positions_ * shape_.width * 4);
    }

private:
    std::vector<std::string> required_names() const {
        std::vector<std::string> names = {"model.encoder.conv1.weight", "model.encoder.conv1.bias",
                                          "model.encoder.conv2.weight", "model.encoder.conv2.bias",
                                          "model.encoder.embed_positions.weight", "model.encoder.layer_norm.weight",
                                          "model.encoder.layer_norm.bias"};
        const char* per_layer[] = {"self_attn.q_proj.weight", "self_attn.q_proj.bias", "self_attn.k_proj.weight",
                                   "self_attn.v_proj.weight", "self_attn.v_proj.bias", "self_attn.out_proj.weight",
                                   "self_attn.out_proj.bias", "self_attn_layer_norm.weight",
                                   "self_attn_layer_norm.bias", "final_layer_norm.weight", "final_layer_norm.bias",
                                   "fc1.weight", "fc1.bias", "fc2.weight", "fc2.bias"};
        for (int l = 0; l < shape_.layers; ++l)
            for (const char* t : per_layer) names.push_back("model.encoder.layers." + std::to_string(l) + "." + t);
        return names;
    }

    void upload_all() {
        for (Vec* v : {&conv1_b_, &conv2_b_, &pos_, &final_w_, &final_b_, &filters_, &window_, &basis_}) v->upload();
        conv1_.upload();
        conv2_.upload();
        for (auto& layer : layers_) {
            Layer& L = *layer;
            for (Vec* v : {&L.ln1_w, &L.ln1_b, &L.qkv_b, &L.o_b, &L.ln2_w, &L.ln2_b, &L.fc1_b, &L.fc2_b}) v->upload();
            for (Product* p : {&L.qkv, &L.o, &L.fc1, &L.fc2}) p->upload();
        }
    }

    void spectrogram(const float* samples, int count) {
        upload_all();
        const int F = shape_.input_frames, M = shape_.mel_bins;
        const size_t window_samples = (size_t)F * kHop;
        // The window's samples, silence past the recording.
        CUDA_CHECK(cudaMemsetAsync(samples_.get(), 0, window_samples * 4, stream_));
        CUDA_CHECK(cudaMemcpyAsync(samples_.get(), samples, (size_t)count * 4, cudaMemcpyDefault, stream_));
        mel_power_kernel<<<F, 256, 0, stream_>>>(samples_.get<float>(), (int)window_samples, window_.get(),
                                                 basis_.get(), power_.get<float>(), F);
        mel_project_kernel<<<dim3((F + 127) / 128, M), 128, 0, stream_>>>(power_.get<float>(), filters_.get(),
                                                                        log_mel_.get<float>(), F);
        max_partials_kernel<<<sm_count_, 256, 0, stream_>>>(log_mel_.get<float>(), M * F, partials_.get<float>());
        mel_normalise_kernel<<<sm_count_, 256, 0, stream_>>>(log_mel_.get<float>(), M * F, partials_.get<float>(),
                                                             sm_count_, mel_.get<float>());
        CUDA_CHECK(cudaGetLastError());
    }

    // One tensor-core product (cross_kv.cuh, linear form): out [rows][p.n] =
    // gelu?(in [rows][p.k] . W^T + bias) (+ residual).
    void product(const float* in, int rows, const Product& p, const float* bias, bool gelu, const float* residual,
                 float* out) {
        CrossKvArgs a{};
        a.encoder = in;
        a.weight = p.device.get();
        a.windows = 1;
        a.rows = rows;
        a.row_stride = rows;
        a.width = p.k;
        a.kblocks = p.kblocks;
        a.columns = p.n;
        a.status = status_.get<int>();
        a.linear_out = out;
        a.bias = bias;
        a.residual = residual;
        a.gelu = gelu ? 1 : 0;
        try {
            launch_cross_kv(storage_ == Storage::f16, a, sm_count_, stream_);
        } catch (const std::runtime_error& e) {
            throw CudaFailure(e.what(), false);
        }
    }

    void layer_norm(const float* in, const Vec& w, const Vec& b, float* out) {
        layer_norm_rows_kernel<<<(positions_ + kNormWarps - 1) / kNormWarps, 32 * kNormWarps, 0, stream_>>>(
            in, w.get(), b.get(), out, positions_, shape_.width);
    }

    // recordEncoder (Encoder.cpp:69-101) and encoderLayer (:34-61).
    void run_encoder() {
        upload_all();
        const int F = shape_.input_frames, M = shape_.mel_bins, d = shape_.width, P = positions_;
        float* columns = columns_.get<float>();
        CUDA_CHECK(cudaMemsetAsync(status_.get(), 0, 16, stream_));
        conv1_columns_kernel<<<4 * sm_count_, 256, 0, stream_>>>(mel_.get<float>(), M, F, columns);
        product(columns, F, conv1_, conv1_b_.get(), true, nullptr, first_.get<float>());
        conv2_columns_kernel<<<4 * sm_count_, 256, 0, stream_>>>(first_.get<float>(), d, F, P, columns);
        // GELU(conv2) + the positional rows, as the product's residual.
        product(columns, P, conv2_, conv2_b_.get(), true, pos_.get(), hidden_.get<float>());
        float* h = hidden_.get<float>();
        for (auto& layer : layers_) {
            Layer& L = *layer;
            layer_norm(h, L.ln1_w, L.ln1_b, normed_.get<float>());
            product(normed_.get<float>(), P, L.qkv, L.qkv_b.get(), false, nullptr, qkv_.get<float>());
            attention_kernel<<<dim3((P + kAttnTile - 1) / kAttnTile, shape_.heads), 256, kAttentionSmem, stream_>>>(
                qkv_.get<float>(), attended_.get<float>(), P, d, 1.f / std::sqrt((float)kHeadWidth));
            product(attended_.get<float>(), P, L.o, L.o_b.get(), false, h, h);
            layer_norm(h, L.ln2_w, L.ln2_b, normed_.get<float>());
            product(normed_.get<float>(), P, L.fc1, L.fc1_b.get(), true, nullptr, ffn_.get<float>());
            product(ffn_.get<float>(), P, L.fc2, L.fc2_b.get(), false, h, h);
        }
        layer_norm(h, final_w_, final_b_, rows_.get<float>());
        CUDA_CHECK(cudaGetLastError());
    }

    void copy_out(float* to, const void* from, size_t bytes) {
        CUDA_CHECK(cudaMemcpyAsync(to, from, bytes, cudaMemcpyDefault, stream_));
        CUDA_CHECK(cudaStreamSynchronize(stream_));
        int status = 0;
        CUDA_CHECK(cudaMemcpy(&status, status_.get(), sizeof(int), cudaMemcpyDeviceToHost));
        if (status != 0)
            throw CudaFailure("an encoder product gave up waiting (wait " + std::to_string(status) + ")", false);
    }

    wsp_encoder_shape shape_;
    int device_ = 0, sm_count_ = 0, positions_ = 0;
    Storage storage_ = Storage::f16;
    cudaStream_t stream_ = nullptr;
    Product conv1_, conv2_;
    Vec conv1_b_, conv2_b_, pos_, final_w_, final_b_, filters_, window_, basis_;
    std::vector<std::unique_ptr<Layer>> layers_;
    std::set<std::string> seen_;
    bool filters_set_ = false;
    DeviceBuffer samples_, power_, log_mel_, mel_, partials_, columns_, first_, hidden_, normed_, qkv_, attended_,
        ffn_, rows_, status_;
};

}  // namespace
}  // namespace wsp

struct wsp_encoder {
    std::unique_ptr<wsp::Encoder> impl;
};

using wsp::guarded;

#define WSP_NEED_ENCODER(e) \
    if (!(e) || !(e)->impl) throw wsp::InvalidArgument("no encoder")

extern "C" {

int wsp_encoder_create(const wsp_encoder_shape* shape, int device, wsp_dtype storage, wsp_encoder** out) {
    return guarded([&] {
        if (!shape || !out) throw wsp::InvalidArgument("wsp_encoder_create needs a shape and an output");
        *out = nullptr;
        auto e = std::make_unique<wsp_encoder>();
        e->impl = std::make_unique<wsp::Encoder>(*shape, device, storage);
        *out = e.release();
    });
}

void wsp_encoder_destroy(wsp_encoder* encoder) { delete encoder; }

int wsp_encoder_set_tensor(wsp_encoder* encoder, const char* name, wsp_dtype dtype, const int64_t* extents,
                           int rank, const void* data) {
    return guarded([&] {
        WSP_NEED_ENCODER(encoder);
        if (!name || (rank > 0 && !extents)) throw wsp::InvalidArgument("a tensor needs a name and its extents");
        encoder->impl->set_tensor(name, dtype, extents, rank, data);
    });
}

int wsp_encoder_set_filters(wsp_encoder* encoder, const float* filters) {
    return guarded([&] {
        WSP_NEED_ENCODER(encoder);
        encoder->impl->set_filters(filters);
    });
}

int wsp_encoder_check_weights(const wsp_encoder* encoder) {
    return guarded([&] {
        WSP_NEED_ENCODER(encoder);
        encoder->impl->check_weights();
    });
}

int wsp_encoder_log_mel(wsp_encoder* encoder, const float* samples, int sample_count, float* mel) {
    return guarded([&] {
        WSP_NEED_ENCODER(encoder);
        encoder->impl->log_mel(samples, sample_count, mel);
    });
}

int wsp_encoder_encode(wsp_encoder* encoder, const float* mel, float* rows) {
    return guarded([&] {
        WSP_NEED_ENCODER(encoder);
        encoder->impl->encode(mel, rows);
    });
}

int wsp_encoder_encode_samples(wsp_encoder* encoder, const float* samples, int sample_count, float* rows) {
    return guarded([&] {
        WSP_NEED_ENCODER(encoder);
        encoder->impl->encode_samples(samples, sample_count, rows);
    });
}

}  // extern "C"
