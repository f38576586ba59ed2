// Stand-ins for the three library types the reference's scalar test decoder
// names, so that decoder can be compiled from its own lines without the
// reference's external dependencies (ea_data_structures, eacp, NanoTest).
// Each stand-in carries only what those lines use: WSP::Vector is
// ea_data_structures' EA::Vector (int size(), operator[], resize), DecoderShape
// the fields and helpers of Lib/WhisperEACP/Decoder/DecoderShape.h:20-83, and
// LayerNorm the epsilon constant of Lib/WhisperEACP/Kernels/LayerNorm.h:21.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <limits>
#include <random>
#include <string>
#include <vector>

namespace WSP
{
template <typename T>
struct Vector : std::vector<T>
{
    using std::vector<T>::vector;
    int size() const { return (int) std::vector<T>::size(); }
};

struct DecoderShape
{
    int width = 0;
    int heads = 0;
    int layers = 0;
    int feedForwardWidth = 0;
    int vocabularySize = 0;
    int maxPositions = 0;
    int crossPositions = 0;

    int headWidth() const { return width / heads; }
    int logitElementCount() const { return vocabularySize; }
    int crossElementCount() const { return crossPositions * width; }
};

struct LayerNorm
{
    static constexpr auto whisperEpsilon = 1e-5f;
};
} // namespace WSP
