// quant.hpp — mirror of the reference include/quant.hpp.
//
// quant_load reads and validates an .abn v2 file exactly as
// src/quant.cpp:31-119 does (magic, version, payload size, FNV-1a checksum);
// an accepted payload is uploaded into the arena, so data and scales are
// DEVICE pointers. A rejected file gives the reference's zeroed block.
#ifndef AAEDN_B200_QUANT_HPP
#define AAEDN_B200_QUANT_HPP

#include <cstddef>
#include <cstdint>

namespace aaedn
{

struct Arena;

enum class QuantType : uint8_t
{
    NONE = 0,
    INT4 = 0,
    INT8 = 1
};

struct QuantBlock
{
    uint8_t* data;    // device: 4-bit codes, low nibble = even element
    uint16_t* scales; // device: one u16 per 32 codes
    size_t num_blocks;
    size_t block_size;
    QuantType type;
    uint32_t format_version;
    uint32_t checksum;
};

QuantBlock quant_load(Arena* arena, const char* path);
void quant_unload(QuantBlock* q);

} // namespace aaedn

#endif
