#!/bin/sh
# Prints, on stdout, one C++ translation unit made of the reference's scalar
# mel spectrogram and scalar encoder, taken from where they lie in the
# reference checkout ($1), between the stand-ins of prelude_frontend.h and
# the C ABI of frontend_abi.inc.  Nothing of the reference is written to
# disk: the Makefile pipes this into g++, and only the compiled library
# lands in oracle/_ref/.
#
#   Tests/Mel/ScalarMel.h      the whole file: periodicHann, reflectPadded,
#                              stftPower, logMel, normalise, melSpectrogram
#   Tests/Kernels/Common.h     20-25 sized
#   Tests/Encoder/Common.h     318-347 ReferenceLayer, ReferenceModel;
#                              390-393 referenceGelu; 398-442 referenceConv1d;
#                              444-507 referenceLayerNorm, referenceLinear;
#                              509-567 referenceAttention; 569-677
#                              referenceEncode; 751-766 syntheticMel
set -eu
ref="$1"
here="$(cd "$(dirname "$0")" && pwd)"
cat "$here/prelude_frontend.h"
cat "$ref/Tests/Mel/ScalarMel.h"
echo "namespace WSP {"
sed -n '20,25p' "$ref/Tests/Kernels/Common.h"
echo "}"
echo "namespace WSP::Testing {"
sed -n '318,347p;390,393p;398,442p;444,507p;509,567p;569,677p;751,766p' "$ref/Tests/Encoder/Common.h"
cat "$here/frontend_abi.inc"
