// dequant.hpp — mirror of the reference include/dequant.hpp. Device
// pointers; asynchronous on the legacy default stream; the u16 scale is cast
// as an integer, as src/dequant.cpp:19 does (bit-exact with it).
#ifndef AAEDN_B200_DEQUANT_HPP
#define AAEDN_B200_DEQUANT_HPP

#include <cstddef>
#include <cstdint>

namespace aaedn
{

void dequant_4bit(const uint8_t* data, const uint16_t* scales, float* output, size_t n);

}

#endif
