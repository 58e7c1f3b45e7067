// attention.hpp — mirror of the reference include/attention.hpp. q, the
// caches and output are device pointers; segments is a HOST array (at most
// 64). Rows of k_cache / v_cache are tokens of n_heads * head_dim floats and
// head h reads its own slice (the reference reads every head from the same
// head_dim floats, src/attention.cpp:40,76).
#ifndef AAEDN_B200_ATTENTION_HPP
#define AAEDN_B200_ATTENTION_HPP

#include <cstddef>
#include <cstdint>

namespace aaedn
{

struct KVCache;
struct Segment;

void attention(const float* q, const float* k_cache, const float* v_cache, const Segment* segments, size_t num_segments,
               float* output, size_t n_heads, size_t head_dim, float scale);

} // namespace aaedn

#endif
