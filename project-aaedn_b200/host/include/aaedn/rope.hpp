// rope.hpp — mirror of the reference include/rope.hpp. rope_init builds the
// reference's table (src/rope.cpp:20-29) on the host and uploads it into the
// arena (device pointers); rope_apply rotates rows 0..seq_len-1 of device q
// and k.
#ifndef AAEDN_B200_ROPE_HPP
#define AAEDN_B200_ROPE_HPP

#include <cstddef>
#include <cstdint>

namespace aaedn
{

struct Arena;

struct RoPETables
{
    float* cos_table; // device [max_seq_len][head_dim/2]
    float* sin_table;
    size_t max_seq_len;
    size_t head_dim;
};

RoPETables rope_init(Arena* arena, size_t max_seq_len, size_t head_dim);
void rope_apply(float* q, float* k, size_t seq_len, size_t head_dim, const RoPETables* tables);

} // namespace aaedn

#endif
