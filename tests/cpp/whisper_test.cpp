// A program that reaches the library only through include/wsp_whisper.hpp:
// Whisper::load on a model directory, its generation config, and (on a GPU)
// prepare + transcribe + transcribeText.
//
//   whisper_test inspect DIR [LANGUAGE [translate]] [-- ID...]
//       load, then print the prompt, the two masks' suppressed ids, the
//       token limit and the hex bytes of decode(ID...)
//   whisper_test refuse DIR
//       load, and print the ModelError's message (exit 1 if none)
//   whisper_test transcribe DIR ENCODER WINDOWS STORAGE CONTEXT
//       load, prepare on device 0 with WINDOWS windows (STORAGE f16 or bf16),
//       set the audio context, transcribe the fp32 rows in ENCODER
//       ([WINDOWS, max_source_positions, d_model]) and print each window's
//       ids and the hex bytes of its text
//   whisper_test context-samples DIR CONTEXT
//       load, set the audio context, and print the ModelError that
//       transcribe_samples raises for a reduced one (exit 1 if none)
//   whisper_test samples DIR AUDIO WINDOWS COUNT
//       load, prepare with WINDOWS windows, transcribe the recordings in
//       AUDIO (WINDOWS x COUNT fp32 samples) through the spectrogram and the
//       encoder, and print each window's ids and the hex bytes of its text
#include "wsp_whisper.hpp"

#include <cstdio>
#include <fstream>
#include <string>
#include <vector>

namespace {

void print_ids(const char* label, const std::vector<uint32_t>& ids) {
    std::printf("%s:", label);
    for (uint32_t id : ids) std::printf(" %u", id);
    std::printf("\n");
}

void print_mask(const char* label, const std::vector<float>& mask) {
    std::printf("%s:", label);
    for (size_t i = 0; i < mask.size(); ++i)
        if (mask[i] != 0.f) std::printf(" %zu", i);
    std::printf("\n");
}

void print_hex(const char* label, const std::string& text) {
    std::printf("%s:", label);
    for (unsigned char c : text) std::printf("%02x", c);
    std::printf("\n");
}

int inspect(int argc, char** argv) {
    wsp::Whisper whisper;
    whisper.load(argv[2]);
    int i = 3;
    if (i < argc && std::string(argv[i]) != "--") {
        const std::string language = argv[i++];
        const bool translate = i < argc && std::string(argv[i]) == "translate";
        if (translate) ++i;
        whisper.set_language(language, translate);
    }
    std::vector<uint32_t> ids;
    if (i < argc && std::string(argv[i]) == "--")
        for (++i; i < argc; ++i) ids.push_back((uint32_t)std::stoul(argv[i]));
    const wsp::ModelConfig& c = whisper.config();
    std::printf("shape: %d %d %d %d %d %d %d\n", c.width, c.decoder_heads, c.decoder_layers, c.decoder_ffn,
                c.vocabulary, c.max_target_positions, c.max_source_positions);
    print_ids("prompt", whisper.prompt());
    print_mask("first", whisper.first_step_suppression());
    print_mask("later", whisper.later_step_suppression());
    std::printf("maximum: %d\n", whisper.maximum_tokens());
    std::printf("context: %d %d %d\n", wsp::Whisper::audio_context_for_samples(16000),
                wsp::Whisper::audio_context_for_samples(20 * 16000),
                wsp::Whisper::audio_context_for_samples(40 * 16000));
    print_hex("text", whisper.tokenizer().decode(ids));
    return 0;
}

int refuse(char** argv) {
    try {
        wsp::Whisper whisper;
        whisper.load(argv[2]);
    } catch (const wsp::ModelError& e) {
        std::printf("refused: %s\n", e.what());
        return 0;
    }
    std::printf("loaded\n");
    return 1;
}

int transcribe(char** argv) {
    wsp::Whisper whisper;
    whisper.load(argv[2]);
    const int windows = std::stoi(argv[4]);
    const wsp_dtype storage = std::string(argv[5]) == "bf16" ? WSP_BFLOAT16 : WSP_FLOAT16;
    const wsp::ModelConfig& c = whisper.config();
    std::vector<float> rows((size_t)windows * c.max_source_positions * c.width);
    std::ifstream in(argv[3], std::ios::binary);
    in.read(reinterpret_cast<char*>(rows.data()), (std::streamsize)(rows.size() * sizeof(float)));
    if (!in) {
        std::printf("short encoder file\n");
        return 1;
    }
    try {
        whisper.transcribe(rows.data());
        std::printf("transcribed before prepare\n");
        return 1;
    } catch (const wsp::ModelError&) {
    }
    whisper.prepare(0, windows, storage);
    whisper.set_audio_context(std::stoi(argv[6]));
    const auto ids = whisper.transcribe(rows.data());
    const auto texts = whisper.transcribe_text(rows.data());
    for (int b = 0; b < windows; ++b) {
        print_ids("ids", ids[b]);
        print_hex("text", texts[b]);
    }
    try {
        whisper.set_audio_context(c.max_source_positions + 1);
        std::printf("accepted an audio context past the window\n");
        return 1;
    } catch (const wsp::ModelError&) {
    }
    std::printf("ok\n");
    return 0;
}

int context_samples(char** argv) {
    wsp::Whisper whisper;
    whisper.load(argv[2]);
    whisper.set_audio_context(std::stoi(argv[3]));
    try {
        whisper.transcribe_samples({});
    } catch (const wsp::ModelError& e) {
        std::printf("refused: %s\n", e.what());
        return 0;
    }
    std::printf("accepted\n");
    return 1;
}

int samples(char** argv) {
    wsp::Whisper whisper;
    whisper.load(argv[2]);
    const int windows = std::stoi(argv[4]), count = std::stoi(argv[5]);
    std::vector<std::vector<float>> recordings((size_t)windows, std::vector<float>((size_t)count));
    std::ifstream in(argv[3], std::ios::binary);
    for (auto& r : recordings) in.read(reinterpret_cast<char*>(r.data()), (std::streamsize)(r.size() * sizeof(float)));
    if (!in) {
        std::printf("short audio file\n");
        return 1;
    }
    whisper.prepare(0, windows);
    if (!whisper.has_front_end()) {
        std::printf("no front end\n");
        return 1;
    }
    const auto ids = whisper.transcribe_samples(recordings);
    const auto texts = whisper.transcribe_samples_text(recordings);
    for (int b = 0; b < windows; ++b) {
        print_ids("ids", ids[b]);
        print_hex("text", texts[b]);
    }
    try {
        recordings.pop_back();
        whisper.transcribe_samples(recordings);
        std::printf("accepted too few recordings\n");
        return 1;
    } catch (const wsp::ModelError&) {
    }
    std::printf("ok\n");
    return 0;
}

}  // namespace

int main(int argc, char** argv) {
    if (argc < 3) {
        std::printf("usage: whisper_test inspect|refuse|transcribe|samples|context-samples DIR ...\n");
        return 2;
    }
    const std::string mode = argv[1];
    try {
        if (mode == "inspect") return inspect(argc, argv);
        if (mode == "refuse") return refuse(argv);
        if (mode == "transcribe" && argc >= 7) return transcribe(argv);
        if (mode == "samples" && argc >= 6) return samples(argv);
        if (mode == "context-samples" && argc >= 4) return context_samples(argv);
    } catch (const std::exception& e) {
        std::printf("error: %s\n", e.what());
        return 1;
    }
    std::printf("bad arguments\n");
    return 2;
}
