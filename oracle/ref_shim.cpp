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
#include "tokenizer.hpp"

#include <algorithm>
#include <cstring>
#include <string>
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

// include/tokenizer.hpp:31-33 — loads path, then (when it loaded) encodes
// text and decodes the ids it got. Returns 1 when the loader accepted the
// file; info[5] = vocab_size, merge_count, max_token_bytes, format_version,
// payload_checksum; ids / bytes capped at their capacities, counts in
// *n_ids / *n_bytes.
int ref_tokenizer(const char* path, const char* text, int add_bos, uint32_t* info, uint32_t* ids, size_t ids_cap,
                  size_t* n_ids, char* bytes, size_t bytes_cap, size_t* n_bytes)
{
    Arena a = arena_create(size_t(64) << 20, 64);
    Tokenizer t = tokenizer_load(&a, path);
    info[0] = t.vocab_size;
    info[1] = t.merge_count;
    info[2] = t.max_token_bytes;
    info[3] = t.format_version;
    info[4] = t.payload_checksum;
    const int ok = t.strings != nullptr;
    *n_ids = 0;
    *n_bytes = 0;
    if (ok && text)
    {
        std::vector<uint32_t> v = tokenizer_encode(&t, text, add_bos != 0);
        *n_ids = v.size();
        std::memcpy(ids, v.data(), std::min(v.size(), ids_cap) * 4);
        std::string d = tokenizer_decode(&t, v);
        *n_bytes = d.size();
        std::memcpy(bytes, d.data(), std::min(d.size(), bytes_cap));
    }
    arena_destroy(&a);
    return ok;
}

// include/tokenizer.hpp:33 on given ids
size_t ref_tokenizer_decode(const char* path, const uint32_t* ids, size_t n, char* bytes, size_t bytes_cap)
{
    Arena a = arena_create(size_t(64) << 20, 64);
    Tokenizer t = tokenizer_load(&a, path);
    std::string d = tokenizer_decode(&t, std::vector<uint32_t>(ids, ids + n));
    std::memcpy(bytes, d.data(), std::min(d.size(), bytes_cap));
    arena_destroy(&a);
    return d.size();
}

} // extern "C"
