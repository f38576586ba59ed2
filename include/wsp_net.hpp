/*
 * wsp_net.hpp -- a CUDA backend behind WhisperEACP's Net op interface, for
 * the decoder: the ops recordSequenceStart and recordDecoderStep
 * (Lib/WhisperEACP/Decoder/Decoder.cpp:121-177) record are lowered onto the
 * C ABI of wsp_decoder.h, header only.
 *
 * wsp::net::Net restates the interface of Lib/WhisperEACP/Net/Net.h:110-171
 * (the same fourteen ops, argument meanings and Tensor/Cache/Binding roles)
 * with this library's plain types in place of eacp's: a Binding is a
 * pointer and a byte count instead of an eacp::GPU::BufferRange, and a
 * Weight is a TensorBuffer's checkpoint name, extents and host bytes
 * (Model/SafeTensors.h:53-65).  A maintainer swaps these for the
 * reference's own types; CudaNet's logic stays as it is.
 *
 * CudaNet records the ops as they come -- a backend may defer and fuse
 * (Net.h:15-18) -- and recognises the decoder's sequence in them: each op
 * checks that its operands are what the decoder passes at that point
 * (their provenance and the weights' HF names), so anything else is
 * refused with wsp::ModelError before it reaches the device.
 *   - Weights are uploaded under their names the first time an op names
 *     them (wsp_decoder_set_tensor).
 *   - The cross-cache appends of recordSequenceStart are the sequence start:
 *     it runs (wsp_decoder_begin_sequence over the encoder rows' binding,
 *     which holds the decoder's cross_positions rows as the encoder's output
 *     buffer does) with the first decoder step after it, once every weight
 *     has been seen, so those rows must stay valid until that step.
 *   - output() of the tied logits completes a decoder step: one
 *     wsp_decoder_step into the logits binding (and the hidden-state binding
 *     if the normalised rows were output first).
 * The encoder's ops (conv1d, transpose, add, a bidirectional attention over
 * encoder rows) are outside this backend and raise wsp::ModelError.
 */
#ifndef WSP_NET_HPP
#define WSP_NET_HPP

#include "wsp_decoder.hpp"

#include <cstdlib>
#include <initializer_list>
#include <map>
#include <string>
#include <vector>

namespace wsp {
namespace net {

enum class Activation { none, gelu };
enum class DType { float32, float16, int32 };

/* A checkpoint tensor: name, extents and host bytes of the given type. */
struct Weight {
    std::string name;
    std::vector<int> shape;
    const void* data = nullptr;
    wsp_dtype type = WSP_FLOAT32;
};

class Shape {
public:
    static constexpr int maxRank = 4;
    Shape() = default;
    Shape(std::initializer_list<int> extents) {
        for (int e : extents)
            if (count_ < maxRank) extents_[count_++] = e;
    }
    int rank() const { return count_; }
    int operator[](int axis) const { return extents_[axis]; }
    int rows() const { return count_ == 0 ? 0 : (count_ == 1 ? 1 : elementCount() / extents_[count_ - 1]); }
    int columns() const { return count_ == 0 ? 0 : extents_[count_ - 1]; }
    int elementCount() const {
        int n = count_ == 0 ? 0 : 1;
        for (int i = 0; i < count_; ++i) n *= extents_[i];
        return n;
    }

private:
    int extents_[maxRank] = {0, 0, 0, 0};
    int count_ = 0;
};

/* Storage outside the net (Net.h:57-69): host or device memory. */
struct Binding {
    void* data = nullptr;
    size_t bytes = 0;
    Shape capacity;
    std::string name;
};

/* Rows a sequence keeps between recordings (Net.h:71-79). */
struct Cache {
    int id = -1;
    int rows = 0;
    void clear() { rows = 0; }
};

class Net;

/* A value inside one recording (Net.h:81-106): copies share it; the net
   reclaims it once the last copy is gone. */
class Tensor {
public:
    Tensor() = default;
    Tensor(Net& owner, int index);
    Tensor(const Tensor& other) : owner_(other.owner_), id_(other.id_) { retain(); }
    Tensor(Tensor&& other) noexcept : owner_(other.owner_), id_(other.id_) {
        other.owner_ = nullptr;
        other.id_ = -1;
    }
    Tensor& operator=(const Tensor& other) {
        if (this != &other) {
            other.retain();
            release();
            owner_ = other.owner_;
            id_ = other.id_;
        }
        return *this;
    }
    Tensor& operator=(Tensor&& other) noexcept {
        if (this != &other) {
            release();
            owner_ = other.owner_;
            id_ = other.id_;
            other.owner_ = nullptr;
            other.id_ = -1;
        }
        return *this;
    }
    ~Tensor() { release(); }
    bool isValid() const { return owner_ != nullptr; }
    bool isOwnedBy(const Net& net) const { return owner_ == &net; }
    int index() const { return id_; }

private:
    void retain() const;
    void release() const;
    Net* owner_ = nullptr;
    int id_ = -1;
};

/* The op interface of Net.h:110-171. */
class Net {
public:
    virtual ~Net() = default;
    virtual Tensor input(const Binding& source, const Shape& shape, DType type) = 0;
    virtual void output(const Tensor& value, const Binding& target) = 0;
    virtual Tensor rows(const Weight& table, int first, int count) = 0;
    virtual Tensor transpose(const Tensor& matrix) = 0;
    virtual Tensor cached(const Cache& cache) = 0;
    virtual Tensor conv1d(const Tensor& frames, const Weight& weight, const Weight& bias, int stride, int padding,
                          Activation activation) = 0;
    virtual Tensor linear(const Tensor& input, const Weight& weight, const Weight* bias, Activation activation) = 0;
    virtual Tensor linearAdd(const Tensor& input, const Weight& weight, const Weight* bias, const Tensor& stream) = 0;
    virtual Tensor add(const Tensor& stream, const Tensor& addend) = 0;
    virtual Tensor layerNorm(const Tensor& input, const Weight& weight, const Weight& bias) = 0;
    virtual Tensor attention(const Tensor& queries, const Tensor& keys, const Tensor& values, int heads,
                             bool causal) = 0;
    virtual Tensor embed(const Tensor& tokens, const Weight& tokenTable, const Weight& positionTable,
                         int firstPosition) = 0;
    virtual Tensor appendLinear(Cache& cache, const Tensor& input, const Weight& weight, const Weight* bias) = 0;
    virtual Cache makeCache(int capacityRows, int width) = 0;

protected:
    friend class Tensor;
    virtual void retain(int index) = 0;
    virtual void release(int index) = 0;
};

inline Tensor::Tensor(Net& owner, int index) : owner_(&owner), id_(index) { retain(); }
inline void Tensor::retain() const {
    if (owner_) owner_->retain(id_);
}
inline void Tensor::release() const {
    if (owner_) owner_->release(id_);
}

/*
 * The CUDA decoder behind Net.  One window; the decoder's shape and storage
 * are given up front (KernelNet sizes its scratch from the same shape).
 */
class CudaNet final : public Net {
public:
    CudaNet(const DecoderShape& shape, int device, wsp_dtype storage = WSP_FLOAT16)
        : shape_(shape), decoder_(shape, device, 1, storage) {}

    CudaDecoder& decoder() { return decoder_; }

    Tensor input(const Binding& source, const Shape& shape, DType type) override {
        if (type == DType::int32 && shape.rank() == 1) {
            if (source.bytes < (size_t)shape[0] * 4) refuse("a token binding smaller than its tokens");
            return make({Tag::tokens, -1, -1, source.data, shape[0]});
        }
        if (type == DType::float32 && shape.rank() == 2 && shape[1] == shape_.width) {
            // The encoder's output buffer: the decoder reads cross_positions
            // rows from it (the first `shape[0]` attended).
            encoder_bytes_ = source.bytes;
            return make({Tag::encoder, -1, -1, source.data, shape[0]});
        }
        refuse("an input that is neither token ids nor encoder rows");
    }

    void output(const Tensor& value, const Binding& target) override {
        const Node& v = node(value);
        if (v.tag == Tag::norm && v.layer == shape_.layers && v.part == kFinal) {
            if (target.bytes < (size_t)v.rows * shape_.width * sizeof(float))
                refuse("a hidden-state binding too small for the step");
            hidden_target_ = static_cast<float*>(target.data);
            return;
        }
        if (v.tag != Tag::logits) refuse("an output other than the decoder's hidden states or logits");
        run_step(target);
    }

    Tensor rows(const Weight&, int, int) override { refuse("rows (an encoder op)"); }
    Tensor transpose(const Tensor&) override { refuse("transpose (an encoder op)"); }
    Tensor conv1d(const Tensor&, const Weight&, const Weight&, int, int, Activation) override {
        refuse("conv1d (an encoder op)");
    }
    Tensor add(const Tensor&, const Tensor&) override { refuse("add (an encoder op)"); }

    Tensor cached(const Cache& cache) override {
        const CacheInfo& c = cache_info(cache);
        if (c.role != Role::cross_keys && c.role != Role::cross_values)
            refuse("cached() of a cache the sequence start did not fill");
        return make({c.role == Role::cross_keys ? Tag::cross_keys : Tag::cross_values, c.layer, -1, nullptr, 0});
    }

    Tensor embed(const Tensor& tokens, const Weight& tokenTable, const Weight& positionTable,
                 int firstPosition) override {
        const Node& t = node(tokens);
        if (t.tag != Tag::tokens) refuse("embed() of something other than token ids");
        expect(tokenTable, "model.decoder.embed_tokens.weight");
        expect(positionTable, "model.decoder.embed_positions.weight");
        const int at = pending_start_ ? 0 : decoder_.position();
        if (firstPosition != at)
            refuse("embed() at position " + std::to_string(firstPosition) + " while the sequence stands at " +
                   std::to_string(at));
        step_tokens_ = static_cast<const uint32_t*>(t.data);
        step_count_ = t.rows;
        hidden_target_ = nullptr;
        return make({Tag::hidden, 0, kLayerInput, nullptr, t.rows});
    }

    Tensor layerNorm(const Tensor& input, const Weight& weight, const Weight& bias) override {
        const Node& x = node(input);
        if (x.tag != Tag::hidden) refuse("a layer norm of something other than the residual stream");
        int part;
        std::string prefix;
        if (x.layer == shape_.layers && x.part == kLayerInput) {
            part = kFinal;
            prefix = "model.decoder.layer_norm";
        } else {
            static const char* const names[] = {"self_attn_layer_norm", "encoder_attn_layer_norm",
                                                "final_layer_norm"};
            part = x.part;  // kLayerInput -> self, kAfterSelf -> cross, kAfterCross -> feed-forward
            prefix = layer_name(x.layer) + names[part];
        }
        expect(weight, prefix + ".weight");
        expect(bias, prefix + ".bias");
        return make({Tag::norm, x.layer, part, nullptr, x.rows});
    }

    Tensor linear(const Tensor& input, const Weight& weight, const Weight* bias, Activation activation) override {
        const Node& x = node(input);
        if (x.tag != Tag::norm) refuse("a projection of something other than normalised rows");
        if (x.part == kFinal) {
            // The tied logits (Decoder.cpp:174-176): embed_tokens, no bias.
            expect(weight, "model.decoder.embed_tokens.weight");
            if (bias || activation != Activation::none) refuse("logits with a bias or an activation");
            return make({Tag::logits, x.layer, -1, nullptr, x.rows});
        }
        const std::string p = layer_name(x.layer);
        if (x.part == kLayerInput || x.part == kAfterSelf) {
            const std::string a = x.part == kLayerInput ? "self_attn" : "encoder_attn";
            expect(weight, p + a + ".q_proj.weight");
            expect_bias(bias, p + a + ".q_proj.bias");
            if (activation != Activation::none) refuse("a query projection with an activation");
            return make({Tag::queries, x.layer, x.part, nullptr, x.rows});
        }
        expect(weight, p + "fc1.weight");
        expect_bias(bias, p + "fc1.bias");
        if (activation != Activation::gelu) refuse("fc1 without its GELU");
        return make({Tag::feed_forward, x.layer, -1, nullptr, x.rows});
    }

    Tensor appendLinear(Cache& cache, const Tensor& input, const Weight& weight, const Weight* bias) override {
        const Node& x = node(input);
        CacheInfo& c = cache_info(cache);
        if (x.tag == Tag::encoder) {
            // recordSequenceStart (Decoder.cpp:121-146): a layer's cross keys
            // or values from the encoder rows.
            const int layer = layer_of(weight.name, "encoder_attn.");
            const bool keys = weight.name == layer_name(layer) + "encoder_attn.k_proj.weight";
            expect(weight, layer_name(layer) + (keys ? "encoder_attn.k_proj.weight" : "encoder_attn.v_proj.weight"));
            if (keys) {
                if (bias) refuse("a cross k_proj with a bias");
            } else {
                expect_bias(bias, layer_name(layer) + "encoder_attn.v_proj.bias");
            }
            c.role = keys ? Role::cross_keys : Role::cross_values;
            c.layer = layer;
            if (cache.rows != 0) refuse("a cross cache appended to twice");
            if (x.rows > shape_.cross_positions)
                throw ModelError("a decoder built for " + std::to_string(shape_.cross_positions) +
                                 " encoder rows was given " + std::to_string(x.rows));
            if (encoder_bytes_ < (size_t)shape_.cross_positions * shape_.width * sizeof(float))
                refuse("an encoder binding that does not hold the decoder's " +
                       std::to_string(shape_.cross_positions) + " rows");
            cache.rows = x.rows;
            sequence_rows_ = static_cast<const float*>(x.data);
            sequence_count_ = x.rows;
            if (++cross_appends_ == 2 * shape_.layers) {
                pending_start_ = true;
                cross_appends_ = 0;
            }
            return make({keys ? Tag::cross_keys : Tag::cross_values, layer, -1, nullptr, x.rows});
        }
        if (x.tag != Tag::norm || x.part != kLayerInput)
            refuse("a cache append of something other than the self attention's normalised rows");
        const std::string p = layer_name(x.layer);
        const bool keys = weight.name == p + "self_attn.k_proj.weight";
        expect(weight, p + (keys ? "self_attn.k_proj.weight" : "self_attn.v_proj.weight"));
        if (keys) {
            if (bias) refuse("a self k_proj with a bias");
        } else {
            expect_bias(bias, p + "self_attn.v_proj.bias");
        }
        c.role = keys ? Role::self_keys : Role::self_values;
        c.layer = x.layer;
        if (cache.rows + x.rows > shape_.max_positions)
            throw ModelError("the self-attention cache holds " + std::to_string(shape_.max_positions) + " rows");
        cache.rows += x.rows;
        return make({keys ? Tag::self_keys : Tag::self_values, x.layer, -1, nullptr, x.rows});
    }

    Tensor attention(const Tensor& queries, const Tensor& keys, const Tensor& values, int heads,
                     bool causal) override {
        const Node& q = node(queries);
        const Node& k = node(keys);
        const Node& v = node(values);
        if (heads != shape_.heads) refuse("attention with " + std::to_string(heads) + " heads");
        if (q.tag != Tag::queries) refuse("attention over something other than projected queries");
        const bool self = q.part == kLayerInput;
        const Tag want_k = self ? Tag::self_keys : Tag::cross_keys, want_v = self ? Tag::self_values : Tag::cross_values;
        if (k.tag != want_k || v.tag != want_v || k.layer != q.layer || v.layer != q.layer || causal != self)
            refuse("attention whose keys, values or mask are not the decoder's");
        return make({Tag::attended, q.layer, q.part, nullptr, q.rows});
    }

    Tensor linearAdd(const Tensor& input, const Weight& weight, const Weight* bias, const Tensor& stream) override {
        const Node& x = node(input);
        const Node& h = node(stream);
        if (h.tag != Tag::hidden || h.layer != x.layer) refuse("a residual add into something other than the stream");
        const std::string p = layer_name(x.layer);
        if (x.tag == Tag::attended) {
            const bool self = x.part == kLayerInput;
            if (h.part != (self ? kLayerInput : kAfterSelf)) refuse("an attention output added out of order");
            const std::string a = self ? "self_attn" : "encoder_attn";
            expect(weight, p + a + ".out_proj.weight");
            expect_bias(bias, p + a + ".out_proj.bias");
            return make({Tag::hidden, x.layer, self ? kAfterSelf : kAfterCross, nullptr, h.rows});
        }
        if (x.tag != Tag::feed_forward || h.part != kAfterCross) refuse("a residual add the decoder does not make");
        expect(weight, p + "fc2.weight");
        expect_bias(bias, p + "fc2.bias");
        return make({Tag::hidden, x.layer + 1, kLayerInput, nullptr, h.rows});
    }

    Cache makeCache(int capacityRows, int width) override {
        if (width != shape_.width) refuse("a cache " + std::to_string(width) + " wide");
        Cache c;
        c.id = (int)caches_.size();
        c.rows = 0;
        caches_.push_back(CacheInfo{Role::unused, -1, capacityRows});
        return c;
    }

protected:
    void retain(int index) override {
        if (index >= 0 && index < (int)nodes_.size()) {
            ++nodes_[index].references;
            ++live_;
        }
    }
    void release(int index) override {
        if (index >= 0 && index < (int)nodes_.size() && nodes_[index].references > 0) {
            --nodes_[index].references;
            if (--live_ == 0) nodes_.clear();  // the recording's values are all gone
        }
    }

private:
    enum class Tag { tokens, encoder, hidden, norm, queries, self_keys, self_values, cross_keys, cross_values,
                     attended, feed_forward, logits };
    enum class Role { unused, self_keys, self_values, cross_keys, cross_values };
    // Where a residual stream value stands in its layer, and which norm.
    static constexpr int kLayerInput = 0, kAfterSelf = 1, kAfterCross = 2, kFinal = 3;

    struct Node {
        Tag tag;
        int layer;
        int part;
        const void* data;  // an input's bound memory
        int rows;
        int references = 0;
    };
    struct CacheInfo {
        Role role;
        int layer;
        int capacity;
    };

    [[noreturn]] static void refuse(const std::string& what) {
        throw ModelError("CudaNet runs the decoder's sequence start and steps; " + what + " does not fit");
    }

    Tensor make(Node n) {
        nodes_.push_back(n);
        return Tensor(*this, (int)nodes_.size() - 1);
    }
    const Node& node(const Tensor& t) const {
        if (!t.isOwnedBy(*this) || t.index() < 0 || t.index() >= (int)nodes_.size())
            refuse("a tensor from another net or recording");
        return nodes_[t.index()];
    }
    CacheInfo& cache_info(const Cache& cache) {
        if (cache.id < 0 || cache.id >= (int)caches_.size()) refuse("a cache this net did not make");
        return caches_[cache.id];
    }
    static std::string layer_name(int layer) { return "model.decoder.layers." + std::to_string(layer) + "."; }
    int layer_of(const std::string& name, const char* part) const {
        const std::string prefix = "model.decoder.layers.";
        if (name.rfind(prefix, 0) != 0) refuse("the weight " + name);
        const size_t dot = name.find('.', prefix.size());
        const int layer = dot == std::string::npos ? -1 : std::atoi(name.substr(prefix.size(), dot - prefix.size()).c_str());
        if (layer < 0 || layer >= shape_.layers || name.find(part, dot) != dot + 1) refuse("the weight " + name);
        return layer;
    }

    // The weight must carry the decoder's name for this place; it is
    // uploaded the first time it is seen.
    void expect(const Weight& w, const std::string& name) {
        if (w.name != name) refuse("the weight " + w.name + " where the decoder reads " + name);
        upload(w);
    }
    void expect_bias(const Weight* w, const std::string& name) {
        if (!w) refuse("no bias where the decoder adds " + name);
        expect(*w, name);
    }
    void upload(const Weight& w) {
        if (uploaded_.count(w.name)) return;
        std::vector<int64_t> extents(w.shape.begin(), w.shape.end());
        decoder_.upload(w.name, w.data, w.type, extents);
        uploaded_[w.name] = true;
    }
    // output() of the logits: the pending sequence start, then the step.
    void run_step(const Binding& logits) {
        if (!step_tokens_) refuse("logits with no step recorded");
        const size_t want = (size_t)step_count_ * shape_.vocabulary_size * sizeof(float);
        if (logits.bytes < want) refuse("a logits binding of " + std::to_string(logits.bytes) + " bytes");
        if (pending_start_) {
            decoder_.checkWeights();
            decoder_.beginSequence(sequence_rows_, sequence_count_);
            pending_start_ = false;
        }
        decoder_.step(step_tokens_, step_count_, static_cast<float*>(logits.data), hidden_target_);
        step_tokens_ = nullptr;
        hidden_target_ = nullptr;
    }

    DecoderShape shape_;
    CudaDecoder decoder_;
    std::vector<Node> nodes_;
    long long live_ = 0;
    std::vector<CacheInfo> caches_;
    std::map<std::string, bool> uploaded_;
    int cross_appends_ = 0;
    bool pending_start_ = false;
    const float* sequence_rows_ = nullptr;
    size_t encoder_bytes_ = 0;
    int sequence_count_ = 0;
    const uint32_t* step_tokens_ = nullptr;
    int step_count_ = 0;
    float* hidden_target_ = nullptr;
};

}  // namespace net
}  // namespace wsp

#endif
