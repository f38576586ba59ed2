// Stand-ins for the library types the reference's scalar encoder names, so
// it can be compiled from its own lines without the reference's external
// dependencies: WSP::Vector (EA::Vector: int size(), operator[]), LayerNorm's
// epsilon (Lib/WhisperEACP/Kernels/LayerNorm.h:21), the output-length rule of
// Lib/WhisperEACP/Kernels/Conv1d.h:119-123, and EncoderShape's fields,
// constants and helpers (Lib/WhisperEACP/Encoder/EncoderShape.h:16-65,
// EncoderShape.cpp:17-32).
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <limits>
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

struct LayerNorm
{
    static constexpr auto whisperEpsilon = 1e-5f;
};

constexpr int conv1dOutputLength(int inputLength, int kernelSize, int stride, int padding)
{
    return (inputLength + 2 * padding - kernelSize) / stride + 1;
}

struct EncoderShape
{
    static constexpr auto convolutionKernelSize = 3;
    static constexpr auto convolutionPadding = 1;
    static constexpr auto firstConvolutionStride = 1;
    static constexpr auto secondConvolutionStride = 2;

    int melBins = 0;
    int width = 0;
    int heads = 0;
    int layers = 0;
    int feedForwardWidth = 0;
    int inputFrames = 0;

    int headWidth() const { return width / heads; }
    int convolutionFrames(int frames) const
    {
        return conv1dOutputLength(frames, convolutionKernelSize, firstConvolutionStride, convolutionPadding);
    }
    int positions(int frames) const
    {
        return conv1dOutputLength(convolutionFrames(frames), convolutionKernelSize, secondConvolutionStride,
                                  convolutionPadding);
    }
    int convolutionFrames() const { return convolutionFrames(inputFrames); }
    int positions() const { return positions(inputFrames); }
    int melElementCount() const { return melBins * inputFrames; }
};
} // namespace WSP
