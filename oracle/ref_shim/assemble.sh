#!/bin/sh
# Prints, on stdout, one C++ translation unit made of the reference's scalar
# test decoder, taken from the lines where they lie in the reference checkout
# ($1), between the stand-ins of prelude.h and the C ABI of ref_abi.inc.
# Nothing of the reference is written to disk: the Makefile pipes this into
# g++, and only the compiled library lands in oracle/_ref/.
#
#   Tests/Kernels/Common.h   20-25 sized, 79-88 spreadValues
#   Tests/Encoder/Common.h   148-156 shiftedValues, 390-393 referenceGelu,
#                            444-507 referenceLayerNorm, referenceLinear
#   Tests/Decoder/Common.h   177-209 the Reference*Weights/Layer/Model structs,
#                            263-500 referenceDecoderAttention, ReferenceDecoding,
#                            referenceDecode, syntheticEncoderOutput, argmaxRow
set -eu
ref="$1"
here="$(cd "$(dirname "$0")" && pwd)"
cat "$here/prelude.h"
echo "namespace WSP {"
sed -n '20,25p;79,88p' "$ref/Tests/Kernels/Common.h"
echo "}"
echo "namespace WSP::Testing {"
sed -n '148,156p;390,393p;444,507p' "$ref/Tests/Encoder/Common.h"
sed -n '177,209p;263,500p' "$ref/Tests/Decoder/Common.h"
echo "}"
cat "$here/ref_abi.inc"
