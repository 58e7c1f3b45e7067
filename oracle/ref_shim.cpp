// ref_shim.cpp — extern "C" entry points over the reference's own C++
// functions, compiled from the reference sources by oracle/Makefile into
// oracle/_ref/libaaedn_ref.so. TEST INFRASTRUCTURE ONLY: it lets the tests
// pin the oracle (oracle.c) against the reference itself. It is never linked
// into the product library.
#include "arena.hpp"
#include "attention.hpp"
#include "dequant.hpp"
#include "ffn.hpp"
#include "kvcache.hpp"
#include "quant.hpp"
#include "rmsnorm.hpp"
#include "rope.hpp"

#include <cstring>
#include <vector>

using namespace aaedn;

extern "C" {

// include/dequant.hpp:10
void ref_dequant_4bit(const uint8_t* data, const uint16_t* scales, float* out, size_t n)
{
    dequant_4bit(data, scales, out, n);
}

// include/rmsnorm.hpp:10
void ref_rmsnorm(const float* in, float* out, const float* w, size_t n, float eps)
{
    rmsnorm(in, out, w, n, eps);
}

// include/rope.hpp:20 — copies the arena tables out
void ref_rope_init(float* cos_out, float* sin_out, size_t max_seq, size_t head_dim)
{
    size_t bytes = max_seq * (head_dim / 2) * sizeof(float);
    Arena a = arena_create(2 * bytes + 4096, 64);
    RoPETables t = rope_init(&a, max_seq, head_dim);
    std::memcpy(cos_out, t.cos_table, bytes);
    std::memcpy(sin_out, t.sin_table, bytes);
    arena_destroy(&a);
}

// include/rope.hpp:21
void ref_rope_apply(float* q, float* k, size_t seq_len, size_t head_dim, float* cos_t, float* sin_t,
                    size_t max_seq)
{
    RoPETables t{cos_t, sin_t, max_seq, head_dim};
    rope_apply(q, k, seq_len, head_dim, &t);
}

// include/attention.hpp:13 — segments given as (start, length) pairs
void ref_attention(const float* q, const float* k, const float* v, const uint32_t* segs, size_t nseg,
                   float* out, size_t n_heads, size_t head_dim, float scale)
{
    std::vector<Segment> s(nseg ? nseg : 1);
    for (size_t i = 0; i < nseg; ++i)
        s[i] = Segment{segs[2 * i], segs[2 * i + 1]};
    attention(q, k, v, segs ? s.data() : nullptr, nseg, out, n_heads, head_dim, scale);
}

// include/ffn.hpp:12 (ffn_dim <= 4096: src/ffn.cpp:10-11 static buffers)
void ref_ffn_swiglu(const float* in, float* out, size_t batch, size_t hidden, size_t ffn, uint8_t* gate,
                    uint8_t* up, uint8_t* down, uint16_t* gs, uint16_t* us, uint16_t* ds)
{
    QuantBlock g{}, u{}, d{};
    g.data = gate;
    g.scales = gs;
    u.data = up;
    u.scales = us;
    d.data = down;
    d.scales = ds;
    ffn_swiglu(in, out, batch, hidden, ffn, &g, &u, &d, gs, us, ds);
}

// include/quant.hpp:30 — 1 when the loader returns data, plus the fields
int ref_quant_load(const char* path, uint64_t* num_blocks, uint32_t* version, uint32_t* checksum)
{
    Arena a = arena_create(size_t(256) << 20, 64);
    QuantBlock q = quant_load(&a, path);
    int ok = q.data != nullptr && q.scales != nullptr;
    *num_blocks = q.num_blocks;
    *version = q.format_version;
    *checksum = q.checksum;
    arena_destroy(&a);
    return ok;
}

} // extern "C"
