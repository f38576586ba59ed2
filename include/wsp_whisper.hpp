/*
 * wsp_whisper.hpp -- WhisperEACP's Whisper::load / prepare / transcribe for the
 * decoder on CUDA, header only, over wsp_decoder.hpp (and through it the C
 * ABI).  It reads a HuggingFace Whisper repository the way the reference does
 * (Lib/WhisperEACP/Whisper/Whisper.cpp:121-146, 148-254):
 *
 *   config.json        ModelConfig (Model/ModelConfig.cpp:57-120): the shape
 *                      fields are required, the generation fields optional
 *   tokenizer.json     the vocabulary and the special tokens
 *                      (Tokenizer/Tokenizer.h:27-80, SpecialTokens.h:17-43)
 *   model.safetensors  the tensors (Model/SafeTensors.h): the decoder's are
 *                      uploaded under their names, the encoder's ignored
 *
 * then builds the generation config: the prompt [decoder_start_token_id (or
 * <|startoftranscript|>), <|notimestamps|>] (buildPrompt, :207-225), the two
 * suppression masks from suppress_tokens and begin_suppress_tokens
 * (buildSuppressionMasks, :227-254) and the token limit max_target_positions -
 * prompt length (:148-154).  A multilingual prompt -- the language and task
 * tokens between the two, which the reference leaves unimplemented
 * (Whisper.h:193-201) -- is setLanguage(code, translate).
 *
 * `transcribe_samples` takes a recording (16 kHz samples, one 30 s window
 * at most) through the log-mel spectrogram and the encoder on CUDA
 * (wsp_encoder.hpp) -- the filterbank is preprocessor_config.json's
 * mel_filters (Model/PreprocessorConfig.cpp:107-135) -- then the greedy
 * search, as Whisper::transcribe does; `transcribe` takes encoder rows
 * ([windows, max_source_positions, d_model] fp32) for a caller with its own
 * encoder.  The _text forms decode the ids with the tokenizer (byte-level
 * BPE, special tokens dropped), as Whisper::transcribeText does
 * (:1497-1507).
 *
 * Errors: wsp::ModelError (a missing file or field, a shape the decoder does
 * not support, a token outside the vocabulary) and the ABI's others.
 */
#ifndef WSP_WHISPER_HPP
#define WSP_WHISPER_HPP

#include "wsp_decoder.hpp"
#include "wsp_encoder.hpp"

#include <cstdint>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <map>
#include <memory>
#include <optional>
#include <sstream>
#include <string>
#include <string_view>
#include <utility>
#include <vector>

namespace wsp {

// ---------------------------------------------------------------------------
// A small JSON reader: enough for config.json, tokenizer.json and a
// safetensors header (objects, arrays, strings with escapes, numbers, true,
// false, null).

namespace json {

struct Value {
    enum Kind { null, boolean, number, string, array, object } kind = null;
    bool b = false;
    double n = 0.0;
    std::string s;
    std::vector<Value> items;
    std::vector<std::pair<std::string, Value>> members;

    const Value* find(std::string_view key) const {
        if (kind != object) return nullptr;
        for (const auto& m : members)
            if (m.first == key) return &m.second;
        return nullptr;
    }
};

class Parser {
public:
    explicit Parser(std::string_view text, std::string what) : t_(text), what_(std::move(what)) {}

    Value document() {
        Value v = value();
        space();
        if (i_ != t_.size()) fail("trailing characters");
        return v;
    }

private:
    [[noreturn]] void fail(const std::string& why) const {
        throw ModelError(what_ + " is not valid JSON (" + why + " at byte " + std::to_string(i_) + ")");
    }
    void space() {
        while (i_ < t_.size() && (t_[i_] == ' ' || t_[i_] == '\n' || t_[i_] == '\r' || t_[i_] == '\t')) ++i_;
    }
    bool take(char c) {
        space();
        if (i_ < t_.size() && t_[i_] == c) {
            ++i_;
            return true;
        }
        return false;
    }
    void expect(char c) {
        if (!take(c)) fail(std::string("expected '") + c + "'");
    }
    bool word(std::string_view w) {
        if (t_.substr(i_, w.size()) == w) {
            i_ += w.size();
            return true;
        }
        return false;
    }
    static void put_utf8(std::string& out, uint32_t cp) {
        if (cp < 0x80) {
            out += (char)cp;
        } else if (cp < 0x800) {
            out += (char)(0xC0 | (cp >> 6));
            out += (char)(0x80 | (cp & 0x3F));
        } else if (cp < 0x10000) {
            out += (char)(0xE0 | (cp >> 12));
            out += (char)(0x80 | ((cp >> 6) & 0x3F));
            out += (char)(0x80 | (cp & 0x3F));
        } else {
            out += (char)(0xF0 | (cp >> 18));
            out += (char)(0x80 | ((cp >> 12) & 0x3F));
            out += (char)(0x80 | ((cp >> 6) & 0x3F));
            out += (char)(0x80 | (cp & 0x3F));
        }
    }
    uint32_t hex4() {
        if (i_ + 4 > t_.size()) fail("a short \\u escape");
        uint32_t v = 0;
        for (int k = 0; k < 4; ++k) {
            const char c = t_[i_++];
            v <<= 4;
            if (c >= '0' && c <= '9') v |= (uint32_t)(c - '0');
            else if (c >= 'a' && c <= 'f') v |= (uint32_t)(c - 'a' + 10);
            else if (c >= 'A' && c <= 'F') v |= (uint32_t)(c - 'A' + 10);
            else fail("a bad \\u escape");
        }
        return v;
    }
    std::string text() {
        expect('"');
        std::string out;
        while (true) {
            if (i_ >= t_.size()) fail("an unterminated string");
            const char c = t_[i_++];
            if (c == '"') return out;
            if (c != '\\') {
                out += c;
                continue;
            }
            if (i_ >= t_.size()) fail("an unterminated escape");
            const char e = t_[i_++];
            switch (e) {
            case '"': out += '"'; break;
            case '\\': out += '\\'; break;
            case '/': out += '/'; break;
            case 'b': out += '\b'; break;
            case 'f': out += '\f'; break;
            case 'n': out += '\n'; break;
            case 'r': out += '\r'; break;
            case 't': out += '\t'; break;
            case 'u': {
                uint32_t cp = hex4();
                if (cp >= 0xD800 && cp < 0xDC00 && word("\\u")) {
                    const uint32_t low = hex4();
                    cp = 0x10000 + ((cp - 0xD800) << 10) + (low - 0xDC00);
                }
                put_utf8(out, cp);
                break;
            }
            default: fail("an unknown escape");
            }
        }
    }
    Value value() {
        space();
        if (i_ >= t_.size()) fail("an unexpected end");
        Value v;
        const char c = t_[i_];
        if (c == '{') {
            ++i_;
            v.kind = Value::object;
            if (take('}')) return v;
            do {
                space();
                std::string key = text();
                expect(':');
                v.members.emplace_back(std::move(key), value());
            } while (take(','));
            expect('}');
        } else if (c == '[') {
            ++i_;
            v.kind = Value::array;
            if (take(']')) return v;
            do v.items.push_back(value());
            while (take(','));
            expect(']');
        } else if (c == '"') {
            v.kind = Value::string;
            v.s = text();
        } else if (word("true")) {
            v.kind = Value::boolean;
            v.b = true;
        } else if (word("false")) {
            v.kind = Value::boolean;
        } else if (word("null")) {
            v.kind = Value::null;
        } else {
            const size_t start = i_;
            while (i_ < t_.size() && std::strchr("+-0123456789.eE", t_[i_]) && t_[i_] != '\0') ++i_;
            if (i_ == start) fail("an unexpected character");
            v.kind = Value::number;
            v.n = std::stod(std::string(t_.substr(start, i_ - start)));
        }
        return v;
    }

    std::string_view t_;
    std::string what_;
    size_t i_ = 0;
};

inline Value parse(std::string_view text, const std::string& what) { return Parser(text, what).document(); }

}  // namespace json

inline std::string read_file(const std::string& path) {
    std::ifstream in(path, std::ios::binary);
    if (!in) throw ModelError("cannot open '" + path + "'");
    std::ostringstream s;
    s << in.rdbuf();
    return s.str();
}

// ---------------------------------------------------------------------------
// config.json: ModelConfig (Model/ModelConfig.h:17-60).

struct ModelConfig {
    int mel_bins = 0, width = 0, encoder_layers = 0, decoder_layers = 0, encoder_heads = 0, decoder_heads = 0;
    int encoder_ffn = 0, decoder_ffn = 0, max_source_positions = 0, max_target_positions = 0, vocabulary = 0;
    static constexpr int no_token = -1;
    int end_of_sequence = no_token, decoder_start = no_token;
    std::vector<int> suppressed, initially_suppressed;

    static ModelConfig from_json(std::string_view text) {
        const json::Value v = json::parse(text, "config.json");
        if (v.kind != json::Value::object) throw ModelError("config.json is not a JSON object");
        if (const json::Value* type = v.find("model_type"))
            if (type->kind != json::Value::string || type->s != "whisper")
                throw ModelError("config.json describes a '" + type->s + "' model, not a whisper one");
        auto integer = [](const json::Value& f, const std::string& what) {
            if (f.kind != json::Value::number) throw ModelError(what + " is not a number");
            if (f.n != (double)(int64_t)f.n) throw ModelError(what + " is not a whole 64-bit integer");
            if (f.n < -2147483648.0 || f.n > 2147483647.0) throw ModelError(what + " does not fit in an int");
            return (int)f.n;
        };
        auto describe = [](const char* field) { return std::string("config.json field '") + field + "'"; };
        auto required = [&](const char* field) {
            const json::Value* f = v.find(field);
            if (!f) throw ModelError(describe(field) + " is missing");
            return integer(*f, describe(field));
        };
        auto optional = [&](const char* field) {
            const json::Value* f = v.find(field);
            return f ? integer(*f, describe(field)) : no_token;
        };
        auto ints = [&](const char* field) {
            std::vector<int> out;
            if (const json::Value* f = v.find(field)) {
                if (f->kind != json::Value::array) throw ModelError(describe(field) + " is not an array");
                for (const json::Value& x : f->items) out.push_back(integer(x, describe(field)));
            }
            return out;
        };
        ModelConfig c;
        const std::pair<const char*, int*> shape[] = {
            {"num_mel_bins", &c.mel_bins},
            {"d_model", &c.width},
            {"encoder_layers", &c.encoder_layers},
            {"decoder_layers", &c.decoder_layers},
            {"encoder_attention_heads", &c.encoder_heads},
            {"decoder_attention_heads", &c.decoder_heads},
            {"encoder_ffn_dim", &c.encoder_ffn},
            {"decoder_ffn_dim", &c.decoder_ffn},
            {"max_source_positions", &c.max_source_positions},
            {"max_target_positions", &c.max_target_positions},
            {"vocab_size", &c.vocabulary},
        };
        for (const auto& f : shape) *f.second = required(f.first);
        c.end_of_sequence = optional("eos_token_id");
        c.decoder_start = optional("decoder_start_token_id");
        c.suppressed = ints("suppress_tokens");
        c.initially_suppressed = ints("begin_suppress_tokens");
        for (const auto& f : shape)
            if (*f.second <= 0) throw ModelError(describe(f.first) + " must be positive");
        if (c.width % c.encoder_heads != 0) throw ModelError("config.json d_model does not divide into the encoder head count");
        if (c.width % c.decoder_heads != 0) throw ModelError("config.json d_model does not divide into the decoder head count");
        return c;
    }

    DecoderShape decoder_shape() const {
        return DecoderShape{width, decoder_heads, decoder_layers, decoder_ffn, vocabulary, max_target_positions,
                            max_source_positions};
    }
};

// ---------------------------------------------------------------------------
// preprocessor_config.json: PreprocessorConfig (Model/PreprocessorConfig.cpp:
// 107-135), the filterbank mel-major [feature_size][n_fft / 2 + 1].

struct PreprocessorConfig {
    int sample_rate = 0, fft_size = 0, hop = 0, mel_bins = 0, chunk_seconds = 0, window_samples = 0, max_frames = 0;
    std::vector<float> mel_filters;

    static PreprocessorConfig from_json(std::string_view text) {
        const json::Value v = json::parse(text, "preprocessor_config.json");
        if (v.kind != json::Value::object) throw ModelError("preprocessor_config.json is not a JSON object");
        auto field = [&](const char* name) {
            const json::Value* f = v.find(name);
            const std::string what = std::string("preprocessor_config.json field '") + name + "'";
            if (!f) throw ModelError(what + " is missing");
            if (f->kind != json::Value::number) throw ModelError(what + " is not a number");
            if (f->n != (double)(int64_t)f->n) throw ModelError(what + " is not a whole 64-bit integer");
            return (int)f->n;
        };
        PreprocessorConfig c;
        c.sample_rate = field("sampling_rate");
        c.fft_size = field("n_fft");
        c.hop = field("hop_length");
        c.mel_bins = field("feature_size");
        c.chunk_seconds = field("chunk_length");
        c.window_samples = field("n_samples");
        c.max_frames = field("nb_max_frames");
        if (c.sample_rate <= 0 || c.hop <= 0 || c.mel_bins <= 0)
            throw ModelError("preprocessor_config.json has a non-positive rate, hop or mel bin count");
        if (c.fft_size <= 0 || c.fft_size % 2 != 0)
            throw ModelError("preprocessor_config.json n_fft is not a positive even number");
        const json::Value* m = v.find("mel_filters");
        if (!m) throw ModelError("preprocessor_config.json field 'mel_filters' is missing");
        if (m->kind != json::Value::array) throw ModelError("preprocessor_config.json mel_filters is not an array");
        const int columns = c.fft_size / 2 + 1;
        int rows = (int)m->items.size(), cols = -1;
        std::vector<float> values;
        for (const json::Value& row : m->items) {
            if (row.kind != json::Value::array)
                throw ModelError("preprocessor_config.json mel_filters has a row that is not an array");
            if (cols < 0) cols = (int)row.items.size();
            else if ((int)row.items.size() != cols) throw ModelError("preprocessor_config.json mel_filters is ragged");
            for (const json::Value& x : row.items) {
                if (x.kind != json::Value::number)
                    throw ModelError("preprocessor_config.json mel_filters is not a number");
                values.push_back((float)x.n);
            }
        }
        if (rows == c.mel_bins && cols == columns) {
            c.mel_filters = std::move(values);
        } else if (rows == columns && cols == c.mel_bins) {
            c.mel_filters.resize(values.size());
            for (int r = 0; r < rows; ++r)
                for (int q = 0; q < cols; ++q) c.mel_filters[(size_t)q * rows + r] = values[(size_t)r * cols + q];
        } else {
            throw ModelError("preprocessor_config.json mel_filters is not " + std::to_string(c.mel_bins) + " x " +
                             std::to_string(columns));
        }
        return c;
    }
};

// ---------------------------------------------------------------------------
// tokenizer.json: the vocabulary's spellings and the special tokens, and
// decoding of ids back to text (Tokenizer.h:27-80, SpecialTokens.h:17-43).

class Tokenizer {
public:
    static Tokenizer from_json(std::string_view text) {
        const json::Value v = json::parse(text, "tokenizer.json");
        const json::Value* model = v.find("model");
        if (!model) throw ModelError("tokenizer.json has no 'model'");
        const json::Value* vocab = model->find("vocab");
        const json::Value* merges = model->find("merges");
        if (!vocab) throw ModelError("tokenizer.json has no 'vocab'");
        if (!merges) throw ModelError("tokenizer.json has no 'merges'");
        if (vocab->kind != json::Value::object) throw ModelError("model.vocab is not an object");
        if (merges->kind != json::Value::array) throw ModelError("model.merges is not an array");
        auto id_of = [](const json::Value& x) {
            if (x.kind != json::Value::number) throw ModelError("tokenizer.json: expected a token id");
            return (int)x.n;
        };
        Tokenizer t;
        for (const auto& m : vocab->members) t.put(m.first, id_of(m.second), false);
        // Every added token counts as special, as Tokenizer::fromJsonText has
        // it (Tokenizer/Tokenizer.cpp:105-160): Whisper's are all <|...|>.
        if (const json::Value* added = v.find("added_tokens"); added && added->kind == json::Value::array)
            for (const json::Value& a : added->items) {
                const json::Value* id = a.find("id");
                const json::Value* content = a.find("content");
                if (!id) throw ModelError("tokenizer.json has no 'id'");
                if (!content) throw ModelError("tokenizer.json has no 'content'");
                t.put(content->s, id_of(*id), true);
            }
        // A spelling names its lowest id.
        for (int id = 0; id < t.size(); ++id)
            if (!t.texts_[id].empty()) t.ids_.emplace(t.texts_[id], id);
        return t;
    }

    int size() const { return (int)texts_.size(); }
    // The vocabulary's own spelling of a token (byte-level alphabet).
    const std::string& text_for(int id) const {
        static const std::string none;
        return id >= 0 && id < size() ? texts_[id] : none;
    }
    bool is_special(int id) const { return id >= 0 && id < size() && special_[id]; }
    int token_for(std::string_view text) const {
        auto it = ids_.find(std::string(text));
        return it == ids_.end() ? ModelConfig::no_token : it->second;
    }

    // The text of the ids, special tokens left out: each token's spelling
    // mapped back through the byte-level alphabet to bytes (UTF-8 text).
    std::string decode(const std::vector<uint32_t>& ids) const {
        std::string bytes;
        for (uint32_t id : ids) {
            if ((int)id >= size() || is_special((int)id)) continue;
            const std::string& s = texts_[id];
            for (size_t i = 0; i < s.size();) {
                uint32_t cp;
                const unsigned char c = (unsigned char)s[i];
                int n = c < 0x80 ? 1 : c < 0xE0 ? 2 : c < 0xF0 ? 3 : 4;
                cp = n == 1 ? c : n == 2 ? (c & 0x1F) : n == 3 ? (c & 0x0F) : (c & 0x07);
                for (int k = 1; k < n && i + k < s.size(); ++k) cp = (cp << 6) | ((unsigned char)s[i + k] & 0x3F);
                i += n;
                const int b = byte_of(cp);
                if (b >= 0) bytes += (char)b;
            }
        }
        return bytes;
    }

private:
    void put(const std::string& text, int id, bool special) {
        if (id < 0) return;
        if (id >= size()) {
            texts_.resize(id + 1);
            special_.resize(id + 1, 0);
        }
        texts_[id] = text;
        special_[id] = special ? 1 : 0;
    }
    // The byte-level alphabet (GPT-2's bytes_to_unicode, which Whisper's
    // tokenizer uses): the printable bytes 33-126, 161-172 and 174-255 stand
    // for themselves, the other 68 bytes for code points 256, 257, ... in
    // byte order.  Returns the byte a code point stands for, or -1.
    static int byte_of(uint32_t cp) {
        auto printable = [](int b) { return (b >= 33 && b <= 126) || (b >= 161 && b <= 172) || (b >= 174 && b <= 255); };
        if (cp < 256) return printable((int)cp) ? (int)cp : -1;
        int n = 256;
        for (int b = 0; b < 256; ++b) {
            if (printable(b)) continue;
            if ((uint32_t)n == cp) return b;
            ++n;
        }
        return -1;
    }

    std::vector<std::string> texts_;
    std::vector<uint8_t> special_;
    std::map<std::string, int> ids_;
};

// ---------------------------------------------------------------------------
// model.safetensors: eight bytes of little-endian header length, the JSON
// header, then the blob the offsets are relative to.

class SafeTensors {
public:
    struct Tensor {
        std::string name;
        wsp_dtype type = WSP_FLOAT32;
        std::vector<int64_t> shape;
        const void* data = nullptr;
    };

    static SafeTensors from_file(const std::string& path) {
        SafeTensors f;
        f.bytes_ = read_file(path);
        if (f.bytes_.size() < 8) throw ModelError(path + " is shorter than a safetensors header");
        uint64_t header = 0;
        for (int i = 7; i >= 0; --i) header = (header << 8) | (unsigned char)f.bytes_[i];
        if (header > f.bytes_.size() - 8) throw ModelError(path + " has a header past its end");
        const json::Value v = json::parse(std::string_view(f.bytes_).substr(8, header), path + " header");
        const size_t blob = 8 + header;
        for (const auto& m : v.members) {
            if (m.first == "__metadata__") continue;
            Tensor t;
            t.name = m.first;
            const json::Value* dtype = m.second.find("dtype");
            const json::Value* shape = m.second.find("shape");
            const json::Value* offsets = m.second.find("data_offsets");
            if (!dtype || !shape || !offsets || offsets->items.size() != 2)
                throw ModelError(path + ": tensor " + t.name + " lacks dtype, shape or data_offsets");
            if (dtype->s == "F32") t.type = WSP_FLOAT32;
            else if (dtype->s == "F16") t.type = WSP_FLOAT16;
            else if (dtype->s == "BF16") t.type = WSP_BFLOAT16;
            else continue;  // not a floating-point weight; not the decoder's
            size_t count = 1;
            for (const json::Value& e : shape->items) {
                t.shape.push_back((int64_t)e.n);
                count *= (size_t)e.n;
            }
            const size_t begin = (size_t)offsets->items[0].n, end = (size_t)offsets->items[1].n;
            const size_t element = t.type == WSP_FLOAT32 ? 4 : 2;
            if (end < begin || blob + end > f.bytes_.size() || end - begin != count * element)
                throw ModelError(path + ": tensor " + t.name + " has data_offsets that do not fit its shape or the file");
            t.data = f.bytes_.data() + blob + begin;
            f.tensors_.push_back(std::move(t));
        }
        return f;
    }

    const std::vector<Tensor>& tensors() const { return tensors_; }

private:
    std::string bytes_;
    std::vector<Tensor> tensors_;
};

// ---------------------------------------------------------------------------

class Whisper {
public:
    // Whisper::load (Whisper.cpp:121-146): the three files of a model
    // directory.
    void load(const std::string& directory) {
        auto require = [&](const char* name) {
            const std::string path = directory + "/" + name;
            if (!std::ifstream(path)) throw ModelError("the model directory " + directory + " has no " + name);
            return path;
        };
        config_ = ModelConfig::from_json(read_file(require("config.json")));
        preprocessor_ = PreprocessorConfig::from_json(read_file(require("preprocessor_config.json")));
        tokenizer_ = Tokenizer::from_json(read_file(require("tokenizer.json")));
        weights_ = std::make_unique<SafeTensors>(SafeTensors::from_file(require("model.safetensors")));
        loaded_ = true;
        language_.clear();
        audio_context_ = 0;
        build_generation_config();
    }
    bool is_loaded() const { return loaded_; }

    // Whisper::prepare: the decoder on a CUDA device, its tensors uploaded
    // and the generation config set.  `windows` windows decode in lockstep.
    // With the checkpoint's encoder tensors, the front end too: the
    // spectrogram's shapes are Whisper's (16 kHz, n_fft 400, hop 160; 80 or
    // 128 mel bins, as config.json and the filterbank agree), which is what
    // Whisper::requireWhisperShapes asks (Whisper.cpp:169-200).
    void prepare(int device = 0, int windows = 1, wsp_dtype storage = WSP_FLOAT16) {
        require_loaded();
        decoder_.reset();
        encoder_.reset();
        auto decoder = std::make_unique<CudaDecoder>(config_.decoder_shape(), device, windows, storage);
        bool has_encoder = false;
        for (const SafeTensors::Tensor& t : weights_->tensors()) {
            if (t.name.rfind("model.decoder.", 0) == 0) decoder->upload(t.name, t.data, t.type, t.shape);
            if (t.name.rfind("model.encoder.conv1.", 0) == 0) has_encoder = true;
        }
        decoder->checkWeights();
        if (has_encoder) {
            if (preprocessor_.mel_bins != config_.mel_bins)
                throw ModelError("this model wants " + std::to_string(config_.mel_bins) +
                                 " mel bins and preprocessor_config.json publishes " +
                                 std::to_string(preprocessor_.mel_bins));
            if (preprocessor_.sample_rate != 16000 || preprocessor_.fft_size != 400 || preprocessor_.hop != 160)
                throw ModelError("preprocessor_config.json describes a front end other than Whisper's "
                                 "(16 kHz, n_fft 400, hop 160)");
            const EncoderShape shape{config_.mel_bins, config_.width, config_.encoder_heads, config_.encoder_layers,
                                     config_.encoder_ffn, 2 * config_.max_source_positions};
            auto encoder = std::make_unique<CudaEncoder>(shape, device, storage);
            for (const SafeTensors::Tensor& t : weights_->tensors())
                if (t.name.rfind("model.encoder.", 0) == 0) encoder->upload(t.name, t.data, t.type, t.shape);
            encoder->setFilters(preprocessor_.mel_filters.data());
            encoder->checkWeights();
            encoder_ = std::move(encoder);
        }
        decoder_ = std::move(decoder);
        apply_generation_config();
    }
    bool has_front_end() const { return encoder_ != nullptr; }
    bool is_prepared() const { return decoder_ != nullptr; }

    const ModelConfig& config() const { return config_; }
    const Tokenizer& tokenizer() const { return tokenizer_; }
    const std::vector<uint32_t>& prompt() const { return prompt_; }
    const std::vector<float>& first_step_suppression() const { return first_mask_; }
    const std::vector<float>& later_step_suppression() const { return later_mask_; }
    int maximum_tokens() const { return maximum_tokens_; }

    // Whisper::setMaximumTokens.
    void set_maximum_tokens(int count) {
        if (count <= 0) throw ModelError("a transcript has to be allowed at least one token");
        maximum_tokens_ = count;
        if (decoder_) apply_generation_config();
    }

    // A multilingual prompt: <|startoftranscript|> <|code|> <|transcribe|> (or
    // <|translate|>) <|notimestamps|>, the form Whisper.h:193-201 describes;
    // an empty code goes back to the two-token prompt.
    void set_language(const std::string& code, bool translate = false) {
        require_loaded();
        language_ = code;
        translate_ = translate;
        build_generation_config();
        if (decoder_) apply_generation_config();
    }

    // Whisper::setAudioContext (Whisper.cpp:415-428): how many of the
    // encoder's positions a run attends to, zero for the whole window.  The
    // encoder rows keep the window's stride; a run reads the first
    // `positions` rows of each window.
    void set_audio_context(int positions) {
        require_loaded();
        if (positions < 0 || positions > config_.max_source_positions)
            throw ModelError("an audio context is between 1 and " + std::to_string(config_.max_source_positions) +
                             " encoder positions, or zero for the whole window, and this one is " +
                             std::to_string(positions));
        audio_context_ = positions;
    }
    int audio_context() const { return audio_context_; }

    // Whisper::audioContextForSamples (Whisper.cpp:450-460): the positions a
    // recording of `samples` 16 kHz samples fills plus `margin_seconds` of
    // what follows, 320 samples a position, rounded up to 64 and held
    // between 448 and the 1500-position window.
    static int audio_context_for_samples(int samples, double margin_seconds = 2.5) {
        const int per_position = 320, tile = 64, floor = 448, window = 1500;
        const int wanted = (samples > 0 ? samples : 0) + (int)(margin_seconds * 16000);
        const int tiles = ((wanted + per_position - 1) / per_position + tile - 1) / tile;
        const int positions = tiles * tile;
        return positions < floor ? floor : positions > window ? window : positions;
    }

    // The greedy search over every window's encoder rows ([windows,
    // max_source_positions, d_model] fp32, host or device): each window's ids,
    // end-of-text excluded.
    std::vector<std::vector<uint32_t>> transcribe(const float* encoder_rows) {
        require_prepared();
        return decoder_->decodeTranscript(encoder_rows, audio_context_);
    }

    // Whisper::transcribeText: the same, decoded to text.
    std::vector<std::string> transcribe_text(const float* encoder_rows) {
        std::vector<std::string> out;
        for (const auto& ids : transcribe(encoder_rows)) out.push_back(tokenizer_.decode(ids));
        return out;
    }

    // Whisper::transcribe on recordings: one per window the decoder was
    // prepared with, each 16 kHz samples of at most one 30 s window (a
    // longer one is a ModelError, as in the reference), through the
    // spectrogram and the encoder, then the greedy search.  Whole windows
    // only: with a reduced audio context the reference's encoder itself
    // computes that many positions from the first twice as many mel frames
    // (Whisper.h:382-402), which this front end does not do yet, so a
    // reduced context here is a ModelError rather than a different answer.
    std::vector<std::vector<uint32_t>> transcribe_samples(const std::vector<std::vector<float>>& recordings) {
        if (audio_context_ != 0 && audio_context_ < config_.max_source_positions)
            throw ModelError("the CUDA front end encodes whole windows, and this Whisper has an audio context of " +
                             std::to_string(audio_context_) + " positions: transcribe encoder rows of that context "
                             "instead, or set the context back to zero");
        require_prepared();
        if (!encoder_) throw ModelError("this model has no encoder tensors: transcribe its encoder rows instead");
        const int windows = decoder_->windows();
        if ((int)recordings.size() != windows)
            throw ModelError("this Whisper decodes " + std::to_string(windows) + " windows at once and was given " +
                             std::to_string(recordings.size()) + " recordings");
        const size_t per = (size_t)encoder_->positions() * config_.width;
        std::vector<float> rows(per * windows);
        for (int b = 0; b < windows; ++b)
            encoder_->encodeSamples(recordings[b].data(), (int)recordings[b].size(), rows.data() + per * b);
        return transcribe(rows.data());
    }
    std::vector<std::string> transcribe_samples_text(const std::vector<std::vector<float>>& recordings) {
        std::vector<std::string> out;
        for (const auto& ids : transcribe_samples(recordings)) out.push_back(tokenizer_.decode(ids));
        return out;
    }

    CudaEncoder& encoder() {
        require_prepared();
        if (!encoder_) throw ModelError("this model has no encoder tensors");
        return *encoder_;
    }

    CudaDecoder& decoder() {
        require_prepared();
        return *decoder_;
    }

private:
    void require_loaded() const {
        if (!loaded_) throw ModelError("this Whisper has not loaded a model yet");
    }
    void require_prepared() const {
        if (!decoder_) throw ModelError("this Whisper has not been prepared on a device yet");
    }

    int special(const char* text) const { return tokenizer_.token_for(text); }

    // buildPrompt and buildSuppressionMasks (Whisper.cpp:207-254).
    void build_generation_config() {
        const int start = config_.decoder_start != ModelConfig::no_token ? config_.decoder_start
                                                                          : special("<|startoftranscript|>");
        if (start == ModelConfig::no_token)
            throw ModelError("neither config.json nor tokenizer.json names <|startoftranscript|>");
        const int no_timestamps = special("<|notimestamps|>");
        if (no_timestamps == ModelConfig::no_token) throw ModelError("tokenizer.json names no <|notimestamps|> token");
        prompt_.assign(1, (uint32_t)start);
        if (!language_.empty()) {
            const int language = special(("<|" + language_ + "|>").c_str());
            const int task = special(translate_ ? "<|translate|>" : "<|transcribe|>");
            if (language == ModelConfig::no_token)
                throw ModelError("tokenizer.json has no language token <|" + language_ + "|>");
            if (task == ModelConfig::no_token) throw ModelError("tokenizer.json has no task token");
            prompt_.push_back((uint32_t)language);
            prompt_.push_back((uint32_t)task);
        }
        prompt_.push_back((uint32_t)no_timestamps);
        const int v = config_.vocabulary;
        auto mark = [v](std::vector<float>& mask, const std::vector<int>& ids) {
            for (int id : ids) {
                if (id < 0 || id >= v)
                    throw ModelError("config.json suppresses token " + std::to_string(id) +
                                     ", which is outside the vocabulary");
                mask[id] = 1.f;
            }
        };
        later_mask_.assign((size_t)v, 0.f);
        mark(later_mask_, config_.suppressed);
        first_mask_ = later_mask_;
        mark(first_mask_, config_.initially_suppressed);
        maximum_tokens_ = config_.max_target_positions - (int)prompt_.size();
        end_of_text_ = config_.end_of_sequence != ModelConfig::no_token ? config_.end_of_sequence
                                                                         : special("<|endoftext|>");
    }

    void apply_generation_config() {
        decoder_->setGeneration(prompt_, first_mask_, later_mask_, maximum_tokens_,
                                (uint32_t)(end_of_text_ < 0 ? 0 : end_of_text_), end_of_text_ >= 0);
    }

    ModelConfig config_;
    PreprocessorConfig preprocessor_;
    Tokenizer tokenizer_;
    std::unique_ptr<SafeTensors> weights_;
    std::unique_ptr<CudaDecoder> decoder_;
    std::unique_ptr<CudaEncoder> encoder_;
    bool loaded_ = false;
    std::vector<uint32_t> prompt_;
    std::vector<float> first_mask_, later_mask_;
    int maximum_tokens_ = 0;
    int end_of_text_ = ModelConfig::no_token;
    std::string language_;
    bool translate_ = false;
    int audio_context_ = 0;
};

}  // namespace wsp

#endif
