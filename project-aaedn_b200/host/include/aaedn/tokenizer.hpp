// tokenizer.hpp — mirror of the reference include/tokenizer.hpp for the B200
// build.
//
// Same names, constants, struct fields and signatures, so callers of the
// reference recompile unchanged. The tables live in HOST memory taken from
// the arena's host part (arena_alloc_host): tokenization is text handling on
// the host around the device token loop. tokenizer_load returns an all-zero
// Tokenizer when the file is rejected (the reference's decisions; the reason
// is aaedn_last_error()). The C ABI (aaedn_tokenizer_*) offers the same
// operations on an opaque handle that keeps its rule table between calls.
#ifndef AAEDN_B200_TOKENIZER_HPP
#define AAEDN_B200_TOKENIZER_HPP

#include <cstddef>
#include <cstdint>
#include <string>
#include <vector>

namespace aaedn
{

struct Arena;

constexpr uint32_t TOKEN_BOS = 32765;
constexpr uint32_t TOKEN_EOS = 32766;
constexpr uint32_t TOKEN_PAD = 32767;

struct Tokenizer
{
    char* strings;           // string block (NUL-terminated strings), host memory
    uint32_t* id_to_offset;  // [vocab_size] offsets into strings
    uint16_t* merges_first;  // [merge_count]
    uint16_t* merges_second; // [merge_count]
    uint32_t vocab_size;
    uint32_t merge_count;
    uint32_t max_token_bytes;
    uint32_t format_version;
    uint32_t payload_checksum;
};

// src/tokenizer.cpp:32-158
Tokenizer tokenizer_load(Arena* arena, const char* path);
// src/tokenizer.cpp:169-239: one id per text byte, merged by the rules;
// TOKEN_BOS first when add_bos
std::vector<uint32_t> tokenizer_encode(const Tokenizer* tok, const char* text, bool add_bos);
// src/tokenizer.cpp:241-257
std::string tokenizer_decode(const Tokenizer* tok, const std::vector<uint32_t>& ids);

} // namespace aaedn

#endif
