// A C++ caller of the library through its C++ headers only: the decoder's
// recording functions, restated from WhisperEACP's Decoder.cpp (the same op
// sequence recordSequenceStart and recordDecoderStep issue against Net,
// Lib/WhisperEACP/Decoder/Decoder.cpp:29-177), run against wsp::net::CudaNet;
// the same inputs through wsp::CudaDecoder directly; and the refusals.
//
//   net_decoder_test <fixture>
//
// The fixture (written by tests/test_gpu_cpp_binding.py) holds a decoder's
// shape and storage, its checkpoint tensors under their HF names, a window's
// encoder rows, a prompt and teacher-forced tokens, and the oracle's logits
// for every position.  Prints the worst errors; exit status 0 when every
// check passes.
#include "wsp_net.hpp"

#include <cmath>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <map>
#include <string>
#include <vector>

namespace {

using wsp::net::Activation;
using wsp::net::Binding;
using wsp::net::Cache;
using wsp::net::DType;
using wsp::net::Net;
using wsp::net::Tensor;
using wsp::net::Weight;

struct Fixture {
    wsp_decoder_shape shape{};
    wsp_dtype storage = WSP_FLOAT16;
    std::map<std::string, Weight> weights;
    std::vector<std::vector<float>> data;  // keeps the tensors' values
    std::vector<float> encoder;            // [cross_positions][width]
    std::vector<uint32_t> prompt, tokens;
    std::vector<float> logits;             // the oracle's, [positions][vocabulary]
};

template <typename T>
T read_one(std::ifstream& in) {
    T v{};
    in.read(reinterpret_cast<char*>(&v), sizeof v);
    if (!in) throw std::runtime_error("fixture truncated");
    return v;
}
template <typename T>
std::vector<T> read_many(std::ifstream& in, size_t n) {
    std::vector<T> v(n);
    in.read(reinterpret_cast<char*>(v.data()), (std::streamsize)(n * sizeof(T)));
    if (!in) throw std::runtime_error("fixture truncated");
    return v;
}

Fixture load(const char* path) {
    std::ifstream in(path, std::ios::binary);
    if (!in) throw std::runtime_error(std::string("cannot open ") + path);
    Fixture f;
    char magic[4];
    in.read(magic, 4);
    if (std::memcmp(magic, "WSPF", 4) != 0) throw std::runtime_error("not a fixture");
    int32_t* fields = &f.shape.width;
    for (int i = 0; i < 7; ++i) fields[i] = read_one<int32_t>(in);
    f.storage = (wsp_dtype)read_one<int32_t>(in);
    const int count = read_one<int32_t>(in);
    f.data.reserve(count);
    for (int t = 0; t < count; ++t) {
        const int name_length = read_one<int32_t>(in);
        std::string name(name_length, '\0');
        in.read(&name[0], name_length);
        const int rank = read_one<int32_t>(in);
        Weight w;
        w.name = name;
        size_t elements = 1;
        for (int r = 0; r < rank; ++r) {
            w.shape.push_back((int)read_one<int64_t>(in));
            elements *= (size_t)w.shape.back();
        }
        f.data.push_back(read_many<float>(in, elements));
        w.data = f.data.back().data();
        w.type = WSP_FLOAT32;
        f.weights[name] = w;
    }
    f.encoder = read_many<float>(in, (size_t)f.shape.cross_positions * f.shape.width);
    f.prompt = read_many<uint32_t>(in, (size_t)read_one<int32_t>(in));
    f.tokens = read_many<uint32_t>(in, (size_t)read_one<int32_t>(in));
    f.logits = read_many<float>(in, (f.prompt.size() + f.tokens.size()) * (size_t)f.shape.vocabulary_size);
    return f;
}

// ---------------------------------------------------------------------------
// The decoder's recording, as Decoder.cpp issues it against Net.

struct LayerWeights {
    const Weight *ln1_w, *ln1_b, *q_w, *q_b, *k_w, *v_w, *v_b, *o_w, *o_b;
    const Weight *ln2_w, *ln2_b, *cq_w, *cq_b, *ck_w, *cv_w, *cv_b, *co_w, *co_b;
    const Weight *ln3_w, *ln3_b, *fc1_w, *fc1_b, *fc2_w, *fc2_b;
};

struct DecoderWeights {
    const Weight *tokens, *positions, *final_w, *final_b;
    std::vector<LayerWeights> layers;
};

struct DecoderCaches {
    std::vector<Cache> self_keys, self_values, cross_keys, cross_values;
};

DecoderWeights bind_weights(const Fixture& f) {
    auto at = [&](const std::string& name) -> const Weight* {
        auto it = f.weights.find(name);
        if (it == f.weights.end()) throw std::runtime_error("fixture lacks " + name);
        return &it->second;
    };
    DecoderWeights w;
    w.tokens = at("model.decoder.embed_tokens.weight");
    w.positions = at("model.decoder.embed_positions.weight");
    w.final_w = at("model.decoder.layer_norm.weight");
    w.final_b = at("model.decoder.layer_norm.bias");
    for (int l = 0; l < f.shape.layers; ++l) {
        const std::string p = "model.decoder.layers." + std::to_string(l) + ".";
        LayerWeights L{};
        L.ln1_w = at(p + "self_attn_layer_norm.weight"); L.ln1_b = at(p + "self_attn_layer_norm.bias");
        L.q_w = at(p + "self_attn.q_proj.weight"); L.q_b = at(p + "self_attn.q_proj.bias");
        L.k_w = at(p + "self_attn.k_proj.weight");
        L.v_w = at(p + "self_attn.v_proj.weight"); L.v_b = at(p + "self_attn.v_proj.bias");
        L.o_w = at(p + "self_attn.out_proj.weight"); L.o_b = at(p + "self_attn.out_proj.bias");
        L.ln2_w = at(p + "encoder_attn_layer_norm.weight"); L.ln2_b = at(p + "encoder_attn_layer_norm.bias");
        L.cq_w = at(p + "encoder_attn.q_proj.weight"); L.cq_b = at(p + "encoder_attn.q_proj.bias");
        L.ck_w = at(p + "encoder_attn.k_proj.weight");
        L.cv_w = at(p + "encoder_attn.v_proj.weight"); L.cv_b = at(p + "encoder_attn.v_proj.bias");
        L.co_w = at(p + "encoder_attn.out_proj.weight"); L.co_b = at(p + "encoder_attn.out_proj.bias");
        L.ln3_w = at(p + "final_layer_norm.weight"); L.ln3_b = at(p + "final_layer_norm.bias");
        L.fc1_w = at(p + "fc1.weight"); L.fc1_b = at(p + "fc1.bias");
        L.fc2_w = at(p + "fc2.weight"); L.fc2_b = at(p + "fc2.bias");
        w.layers.push_back(L);
    }
    return w;
}

Tensor layer(Net& net, const wsp_decoder_shape& shape, const LayerWeights& w, DecoderCaches& c, int index,
             const Tensor& hidden) {
    const Tensor n1 = net.layerNorm(hidden, *w.ln1_w, *w.ln1_b);
    const Tensor q = net.linear(n1, *w.q_w, w.q_b, Activation::none);
    const Tensor k = net.appendLinear(c.self_keys[index], n1, *w.k_w, nullptr);
    const Tensor v = net.appendLinear(c.self_values[index], n1, *w.v_w, w.v_b);
    const Tensor after_self = net.linearAdd(net.attention(q, k, v, shape.heads, true), *w.o_w, w.o_b, hidden);
    const Tensor n2 = net.layerNorm(after_self, *w.ln2_w, *w.ln2_b);
    const Tensor q2 = net.linear(n2, *w.cq_w, w.cq_b, Activation::none);
    const Tensor after_cross =
        net.linearAdd(net.attention(q2, net.cached(c.cross_keys[index]), net.cached(c.cross_values[index]),
                                    shape.heads, false),
                      *w.co_w, w.co_b, after_self);
    const Tensor n3 = net.layerNorm(after_cross, *w.ln3_w, *w.ln3_b);
    return net.linearAdd(net.linear(n3, *w.fc1_w, w.fc1_b, Activation::gelu), *w.fc2_w, w.fc2_b, after_cross);
}

void record_sequence_start(Net& net, const wsp_decoder_shape& shape, const DecoderWeights& w, DecoderCaches& c,
                           const Binding& encoder_rows, int rows) {
    const Tensor encoded = net.input(encoder_rows, {rows, shape.width}, DType::float32);
    for (int l = 0; l < shape.layers; ++l) {
        c.self_keys[l].clear();
        c.self_values[l].clear();
        c.cross_keys[l].clear();
        c.cross_values[l].clear();
        net.appendLinear(c.cross_keys[l], encoded, *w.layers[l].ck_w, nullptr);
        net.appendLinear(c.cross_values[l], encoded, *w.layers[l].cv_w, w.layers[l].cv_b);
    }
}

void record_decoder_step(Net& net, const wsp_decoder_shape& shape, const DecoderWeights& w, DecoderCaches& c,
                         const Binding& tokens, int count, int first, const Binding& hidden_states,
                         const Binding& logits) {
    Tensor hidden = net.embed(net.input(tokens, {count}, DType::int32), *w.tokens, *w.positions, first);
    for (int l = 0; l < shape.layers; ++l) hidden = layer(net, shape, w.layers[l], c, l, hidden);
    const Tensor normalised = net.layerNorm(hidden, *w.final_w, *w.final_b);
    net.output(normalised, hidden_states);
    net.output(net.linear(normalised, *w.tokens, nullptr, Activation::none), logits);
}

// ---------------------------------------------------------------------------

int failures = 0;
void expect(bool ok, const std::string& what) {
    if (!ok) {
        std::printf("FAIL: %s\n", what.c_str());
        ++failures;
    }
}

double max_abs(const float* a, const float* b, size_t n) {
    double worst = 0.0;
    for (size_t i = 0; i < n; ++i) worst = std::fmax(worst, std::fabs((double)a[i] - (double)b[i]));
    return worst;
}

}  // namespace

int main(int argc, char** argv) {
    if (argc != 2) {
        std::fprintf(stderr, "usage: %s <fixture>\n", argv[0]);
        return 2;
    }
    try {
        Fixture f = load(argv[1]);
        const wsp_decoder_shape& shape = f.shape;
        const int V = shape.vocabulary_size, d = shape.width;
        const int P = (int)f.prompt.size(), steps = (int)f.tokens.size();
        DecoderWeights weights = bind_weights(f);

        // 1. The recording through CudaNet.
        wsp::net::CudaNet net(shape, 0, f.storage);
        DecoderCaches caches;
        for (int l = 0; l < shape.layers; ++l) {
            caches.self_keys.push_back(net.makeCache(shape.max_positions, d));
            caches.self_values.push_back(net.makeCache(shape.max_positions, d));
            caches.cross_keys.push_back(net.makeCache(shape.cross_positions, d));
            caches.cross_values.push_back(net.makeCache(shape.cross_positions, d));
        }
        Binding encoder{f.encoder.data(), f.encoder.size() * sizeof(float), {shape.cross_positions, d}, "encoder"};
        record_sequence_start(net, shape, weights, caches, encoder, shape.cross_positions);
        std::vector<float> net_logits((size_t)(P + steps) * V), net_hidden((size_t)(P + steps) * d);
        int position = 0;
        auto run = [&](const uint32_t* ids, int count) {
            Binding tokens{const_cast<uint32_t*>(ids), (size_t)count * 4, {count}, "tokens"};
            Binding hidden{net_hidden.data() + (size_t)position * d, (size_t)count * d * 4, {count, d}, "hidden"};
            Binding logits{net_logits.data() + (size_t)position * V, (size_t)count * V * 4, {count, V}, "logits"};
            record_decoder_step(net, shape, weights, caches, tokens, count, position, hidden, logits);
            position += count;
        };
        run(f.prompt.data(), P);
        for (int k = 0; k < steps; ++k) run(&f.tokens[k], 1);
        expect(net.decoder().position() == P + steps, "the decoder's position after the steps");
        expect(caches.self_keys[0].rows == P + steps, "the self cache's rows after the steps");
        const double net_error = max_abs(net_logits.data(), f.logits.data(), net_logits.size());
        std::printf("CudaNet: %d positions, logits max-abs %.3g against the oracle\n", P + steps, net_error);
        expect(net_error <= 2e-2, "CudaNet logits within max-abs 2e-2 of the oracle");

        // 2. The same inputs through CudaDecoder: the same launches, so the
        //    same bits.
        wsp::CudaDecoder direct(shape, 0, 1, f.storage);
        for (const auto& entry : f.weights) {
            const Weight& w = entry.second;
            direct.upload(w.name, w.data, w.type, std::vector<int64_t>(w.shape.begin(), w.shape.end()));
        }
        direct.checkWeights();
        direct.beginSequence(f.encoder.data());
        std::vector<float> direct_logits((size_t)(P + steps) * V);
        direct.step(f.prompt.data(), P, direct_logits.data());
        for (int k = 0; k < steps; ++k) direct.step(&f.tokens[k], 1, direct_logits.data() + (size_t)(P + k) * V);
        expect(std::memcmp(direct_logits.data(), net_logits.data(), direct_logits.size() * 4) == 0,
               "CudaDecoder and CudaNet give the same logits");

        // 3. Refusals, raised on the host before anything is launched.
        bool refused = false;
        try {
            std::vector<uint32_t> many((size_t)shape.max_positions, 1u);
            direct.step(many.data(), shape.max_positions, nullptr);
        } catch (const wsp::ModelError&) {
            refused = true;
        }
        expect(refused, "a step past max_positions raises ModelError");
        expect(direct.position() == P + steps, "a refused step leaves the position");
        refused = false;
        try {
            net.add(Tensor(), Tensor());
        } catch (const wsp::ModelError&) {
            refused = true;
        }
        expect(refused, "an encoder op on CudaNet raises ModelError");
        refused = false;
        try {
            wsp::CudaDecoder unfinished(shape, 0, 1, f.storage);
            unfinished.checkWeights();
        } catch (const wsp::ModelError& e) {
            refused = std::string(e.what()).find("model.decoder.") != std::string::npos;
        }
        expect(refused, "missing weights are named in a ModelError");
    } catch (const std::exception& e) {
        std::printf("FAIL: %s\n", e.what());
        return 1;
    }
    std::printf("%s\n", failures == 0 ? "ok" : "failed");
    return failures == 0 ? 0 : 1;
}
