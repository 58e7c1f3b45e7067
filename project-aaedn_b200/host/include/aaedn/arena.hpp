// arena.hpp — mirror of the reference include/arena.hpp for the B200 build.
//
// Same names and signatures. An Arena is one device allocation (cudaMalloc
// at arena_create) with a bump pointer, as the reference's single
// pre-allocated arena (src/arena.cpp:7-27); arena_alloc returns DEVICE
// memory. Host-side tables (the KV cache's branch and segment tables, the
// tokenizer's tables) come from a host arena kept beside it (arena_alloc_host;
// as large as the device part, at least 1 MB). Where the
// reference asserts on overflow, arena_alloc returns nullptr and records the
// error (aaedn_last_error()).
#ifndef AAEDN_B200_ARENA_HPP
#define AAEDN_B200_ARENA_HPP

#include <cstddef>
#include <cstdint>

namespace aaedn
{

struct Arena
{
    uint8_t* base; // device memory
    size_t capacity;
    size_t used;
    uint8_t* host_base; // host memory for host-side tables
    size_t host_capacity;
    size_t host_used;
};

Arena arena_create(size_t bytes, size_t align = 32);
void* arena_alloc(Arena* a, size_t bytes, size_t align = 32);
void* arena_alloc_host(Arena* a, size_t bytes, size_t align = 32);
void arena_destroy(Arena* a);

} // namespace aaedn

#endif
