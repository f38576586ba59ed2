// A C ABI over the reference's own fp16 narrowing
// (Lib/WhisperEACP/Core/Utils/Half.cpp), which compiles stand-alone.
#include "Half.h"

extern "C" std::uint16_t ref_pack_half(float value)
{
    return WSP::packHalf(value);
}

extern "C" float ref_half_to_float(std::uint16_t bits)
{
    return WSP::halfToFloat(bits);
}
