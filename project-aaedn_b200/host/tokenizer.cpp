// tokenizer.cpp — the .abt v2 tokenizer around the token loop
// (src/tokenizer.cpp:32-257; the writer is tools/convert_tokenizer.py:44-93):
// file reader, byte-level BPE encode, decode. Host code: text handling has
// no place on the GPU; the token ids it produces feed the decode loop.
//
// File: a 64-byte little-endian header "<8sIQI4I24s" (magic "AAEDNTOK",
// version 2, payload_size u64, FNV-1a 32 of the payload, vocab_size,
// max_token_bytes, merge_count, the payload size again as u32, 24 reserved
// bytes), then the payload: vocab_size, max_token_bytes, merge_count and the
// string-block size (u32 each), the string block (token strings, each
// NUL-terminated), vocab_size u32 offsets into it, merge_count (u16 first,
// u16 second) rules. A file is accepted exactly when the reference's loader
// accepts it (src/tokenizer.cpp:32-158): magic, version 2, the two payload
// sizes equal, the file exactly header + payload, a non-empty payload whose
// checksum matches, the payload's three counts equal to the header's, a
// string block no larger than the payload, and enough payload bytes for the
// block, the offsets and the rules (trailing bytes are allowed).
//
// Encode keeps the reference's merge discipline (src/tokenizer.cpp:169-239),
// because the ids depend on it: one token per input byte; every adjacent
// pair some rule matches (the lowest-numbered rule with that first and
// second) is queued under that rule's number alone; the lowest number is
// popped, skipped when its two tokens are no longer at its position, else
// the pair becomes token vocab_size + rule, the second token is erased, and
// the new pairs on its left and then its right are queued. Entries keep the
// position they were queued at (later erasures shift the tokens under them;
// the same check decides), and entries with equal rule numbers leave the
// queue in the order of the standard library's binary heap, so the queue is
// a std::priority_queue ordered by rule number, as in the reference. What
// differs is the cost, not the result: the reference scans every rule for
// every pair and erases from a vector (O(n) a merge); here a hash table from
// the pair to its lowest rule number, built once per loaded tokenizer,
// answers in O(1), and the sequence is a linked list of byte slots with a
// Fenwick tree that finds the k-th present token in O(log n).
//
// Decode (src/tokenizer.cpp:241-257): ids 32766 (EOS) and 32767 (PAD) and
// ids >= vocab_size contribute nothing, every other id its string. One
// deliberate difference: an offset that points outside the string block
// (which the reference's loader accepts and its decode then reads out of
// bounds) decodes as the empty string here.
#include <cstdio>
#include <cstring>
#include <new>
#include <queue>
#include <string>
#include <unordered_map>
#include <vector>

#include "aaedn/arena.hpp"
#include "aaedn/tokenizer.hpp"
#include "aaedn_b200.h"
#include "host_common.hpp"

using aaedn_host::set_error;

namespace
{

constexpr uint32_t kAbtVersion = 2;       // src/tokenizer.cpp:11
constexpr size_t kAbtHeaderBytes = 64;    // tools/convert_tokenizer.py:11
constexpr uint32_t kBos = 32765, kEos = 32766, kPad = 32767; // include/tokenizer.hpp:15-17

uint32_t rd32(const uint8_t* p) { return (uint32_t)p[0] | (uint32_t)p[1] << 8 | (uint32_t)p[2] << 16 | (uint32_t)p[3] << 24; }
uint64_t rd64(const uint8_t* p) { return (uint64_t)rd32(p) | (uint64_t)rd32(p + 4) << 32; }
uint16_t rd16(const uint8_t* p) { return (uint16_t)(p[0] | p[1] << 8); }

} // namespace

// The decoded tables of one tokenizer (the C ABI's opaque handle).
struct aaedn_tokenizer
{
    uint32_t vocab_size = 0, merge_count = 0, max_token_bytes = 0, format_version = 0, payload_checksum = 0;
    std::vector<char> strings;             // the string block, plus one NUL after it
    std::vector<uint32_t> offsets;         // [vocab_size], each inside the block (else the final NUL)
    std::vector<uint16_t> first, second;   // [merge_count]
    std::unordered_map<uint32_t, uint32_t> rule; // (first << 16 | second) -> lowest rule number
};

namespace
{

// The lowest-numbered rule for each (first, second) pair.
void build_rule_table(const uint16_t* first, const uint16_t* second, uint32_t n,
                      std::unordered_map<uint32_t, uint32_t>& rule)
{
    rule.clear();
    rule.reserve((size_t)n * 2 + 1);
    for (uint32_t m = 0; m < n; ++m)
        rule.emplace((uint32_t)first[m] << 16 | second[m], m); // keeps the first (lowest) m
}

// Parses a whole .abt file image (header + payload) with the reference's
// accept/reject decisions; AAEDN_EFORMAT on rejection.
int parse_abt(const uint8_t* img, size_t n, aaedn_tokenizer& t)
{
    if (n < kAbtHeaderBytes)
        return set_error(AAEDN_EFORMAT, "abt: %zu bytes: shorter than the 64-byte header", n);
    if (std::memcmp(img, "AAEDNTOK", 8) != 0)
        return set_error(AAEDN_EFORMAT, "abt: bad magic");
    const uint32_t version = rd32(img + 8);
    const uint64_t payload_size = rd64(img + 12);
    const uint32_t checksum = rd32(img + 20);
    const uint32_t vocab = rd32(img + 24), max_bytes = rd32(img + 28), merges = rd32(img + 32);
    const uint32_t declared = rd32(img + 36);
    if (version != kAbtVersion)
        return set_error(AAEDN_EFORMAT, "abt: version %u (want %u)", version, kAbtVersion);
    if (payload_size != declared)
        return set_error(AAEDN_EFORMAT, "abt: payload sizes differ (%llu, %u)", (unsigned long long)payload_size,
                         declared);
    if ((uint64_t)(n - kAbtHeaderBytes) != payload_size)
        return set_error(AAEDN_EFORMAT, "abt: file holds %zu payload bytes, header says %llu", n - kAbtHeaderBytes,
                         (unsigned long long)payload_size);
    if (payload_size == 0)
        return set_error(AAEDN_EFORMAT, "abt: empty payload");
    const uint8_t* p = img + kAbtHeaderBytes;
    const uint8_t* e = p + payload_size;
    if (aaedn_fnv1a32(p, (size_t)payload_size, 0x811C9DC5u) != checksum)
        return set_error(AAEDN_EFORMAT, "abt: payload checksum mismatch");
    if (e - p < 16)
        return set_error(AAEDN_EFORMAT, "abt: payload shorter than its four counts");
    const uint32_t pv = rd32(p), pm = rd32(p + 4), pc = rd32(p + 8), block = rd32(p + 12);
    p += 16;
    if (pv != vocab || pm != max_bytes || pc != merges || block > payload_size)
        return set_error(AAEDN_EFORMAT, "abt: payload counts disagree with the header");
    if ((size_t)(e - p) < block)
        return set_error(AAEDN_EFORMAT, "abt: string block truncated");
    const uint8_t* sb = p;
    p += block;
    if ((size_t)(e - p) / 4 < vocab)
        return set_error(AAEDN_EFORMAT, "abt: offsets truncated");
    const uint8_t* ob = p;
    p += (size_t)vocab * 4;
    if ((size_t)(e - p) / 4 < merges)
        return set_error(AAEDN_EFORMAT, "abt: merge rules truncated");
    try
    {
        t.strings.assign(reinterpret_cast<const char*>(sb), reinterpret_cast<const char*>(sb) + block);
        t.strings.push_back('\0'); // a string that runs to the block's end stops here
        t.offsets.resize(vocab);
        for (uint32_t i = 0; i < vocab; ++i)
        {
            const uint32_t off = rd32(ob + 4 * (size_t)i);
            t.offsets[i] = off < block ? off : block; // outside the block: the empty string
        }
        t.first.resize(merges);
        t.second.resize(merges);
        for (uint32_t m = 0; m < merges; ++m)
        {
            t.first[m] = rd16(p + 4 * (size_t)m);
            t.second[m] = rd16(p + 4 * (size_t)m + 2);
        }
        build_rule_table(t.first.data(), t.second.data(), merges, t.rule);
    }
    catch (const std::bad_alloc&)
    {
        return set_error(AAEDN_ENOMEM, "abt: tables do not fit in host memory");
    }
    t.vocab_size = vocab;
    t.merge_count = merges;
    t.max_token_bytes = max_bytes;
    t.format_version = version;
    t.payload_checksum = checksum;
    return AAEDN_OK;
}

int read_file(const char* path, std::vector<uint8_t>& out)
{
    if (!path)
        return set_error(AAEDN_EINVAL, "abt: null path");
    FILE* f = std::fopen(path, "rb");
    if (!f)
        return set_error(AAEDN_EFORMAT, "abt: cannot open %s", path);
    std::fseek(f, 0, SEEK_END);
    const long end = std::ftell(f);
    std::fseek(f, 0, SEEK_SET);
    int rc = AAEDN_OK;
    if (end < 0)
        rc = set_error(AAEDN_EFORMAT, "abt: cannot size %s", path);
    else
    {
        out.resize((size_t)end);
        if (end > 0 && std::fread(out.data(), 1, (size_t)end, f) != (size_t)end)
            rc = set_error(AAEDN_EFORMAT, "abt: short read of %s", path);
    }
    std::fclose(f);
    return rc;
}

// A queued merge: rule number, the position of the pair's first token when
// it was queued, and the pair. Ordered by rule number alone (lowest first).
struct Merge
{
    uint32_t rule;
    uint32_t pos;
    uint16_t a, b;
    bool operator<(const Merge& o) const { return rule > o.rule; }
};

// The token sequence during encode. The queue's positions count the tokens
// present now (an erasure shifts every later one down by one), so a token
// keeps the slot of its first byte, merged-away slots leave a linked list of
// present slots, and a Fenwick tree over the slots finds the slot of the
// k-th present token in O(log n): O((n + merges) log n) for a text of n
// bytes, where erasing from a vector (the reference) costs O(n) a merge.
class TokenSeq
{
  public:
    explicit TokenSeq(const unsigned char* text, size_t n)
        : val_(n), prev_(n), next_(n), bit_(n + 1), n_(n), present_(n)
    {
        for (size_t i = 0; i < n; ++i)
        {
            val_[i] = text[i];
            prev_[i] = (int64_t)i - 1;
            next_[i] = i + 1 < n ? (int64_t)i + 1 : -1;
        }
        for (size_t i = 1; i <= n; ++i) // every slot present: bit[i] = lowbit(i)
            bit_[i] = (uint32_t)(i & (~i + 1));
        top_ = 1;
        while (top_ * 2 <= n)
            top_ *= 2;
    }
    size_t size() const { return present_; }
    uint32_t& val(int64_t slot) { return val_[(size_t)slot]; }
    int64_t prev(int64_t slot) const { return prev_[(size_t)slot]; }
    int64_t next(int64_t slot) const { return next_[(size_t)slot]; }
    // slot of the k-th present token (k < size())
    int64_t slot_of(size_t k) const
    {
        size_t pos = 0, rem = k + 1;
        for (size_t step = top_; step; step >>= 1)
            if (pos + step <= n_ && bit_[pos + step] < rem)
            {
                pos += step;
                rem -= bit_[pos];
            }
        return (int64_t)pos; // the last prefix with fewer than k + 1 present: 0-based slot pos
    }
    void erase(int64_t slot)
    {
        for (size_t i = (size_t)slot + 1; i <= n_; i += i & (~i + 1))
            --bit_[i];
        const int64_t p = prev_[(size_t)slot], q = next_[(size_t)slot];
        if (p >= 0)
            next_[(size_t)p] = q;
        if (q >= 0)
            prev_[(size_t)q] = p;
        --present_;
    }

  private:
    std::vector<uint32_t> val_;
    std::vector<int64_t> prev_, next_;
    std::vector<uint32_t> bit_;
    size_t n_, present_, top_;
};

// Byte-level BPE over a rule table (see the file comment).
std::vector<uint32_t> encode_core(const std::unordered_map<uint32_t, uint32_t>& rule, uint32_t vocab_size,
                                  const char* text, bool add_bos)
{
    const size_t n = std::strlen(text);
    TokenSeq seq(reinterpret_cast<const unsigned char*>(text), n);
    // the rule for tokens (x, y), or false (ids above 16 bits match none)
    auto find = [&](uint32_t x, uint32_t y, uint32_t& m) {
        if ((x | y) > 0xFFFFu)
            return false;
        const auto it = rule.find(x << 16 | y);
        if (it == rule.end())
            return false;
        m = it->second;
        return true;
    };
    std::priority_queue<Merge> q;
    uint32_t m;
    for (size_t i = 0; i + 1 < n; ++i) // every slot is present: slot i is position i
        if (find(seq.val((int64_t)i), seq.val((int64_t)i + 1), m))
            q.push({m, (uint32_t)i, (uint16_t)seq.val((int64_t)i), (uint16_t)seq.val((int64_t)i + 1)});
    while (!q.empty())
    {
        const Merge top = q.top();
        q.pop();
        const size_t p = top.pos;
        if (p + 1 >= seq.size())
            continue;
        const int64_t i = seq.slot_of(p), j = seq.next(i);
        if (seq.val(i) != top.a || seq.val(j) != top.b)
            continue; // stale: the pair is gone or something else sits here now
        seq.val(i) = vocab_size + top.rule;
        seq.erase(j);
        if (p > 0)
        {
            const int64_t h = seq.prev(i);
            if (find(seq.val(h), seq.val(i), m))
                q.push({m, (uint32_t)(p - 1), (uint16_t)seq.val(h), (uint16_t)seq.val(i)});
        }
        if (p + 1 < seq.size())
        {
            const int64_t k = seq.next(i);
            if (find(seq.val(i), seq.val(k), m))
                q.push({m, (uint32_t)p, (uint16_t)seq.val(i), (uint16_t)seq.val(k)});
        }
    }
    std::vector<uint32_t> out;
    out.reserve(seq.size() + (add_bos ? 1 : 0));
    if (add_bos)
        out.push_back(kBos);
    for (int64_t s = n ? 0 : -1; s >= 0; s = seq.next(s)) // slot 0 is never merged away
        out.push_back(seq.val(s));
    return out;
}

// The strings of ids, concatenated (see the file comment). `strings` ends in
// a NUL and every offset lies inside it.
std::string decode_core(const char* strings, const uint32_t* offsets, uint32_t vocab_size, const uint32_t* ids,
                        size_t n)
{
    std::string out;
    if (!strings || !offsets)
        return out;
    for (size_t k = 0; k < n; ++k)
    {
        const uint32_t id = ids[k];
        if (id == kEos || id == kPad || id >= vocab_size)
            continue;
        out += strings + offsets[id];
    }
    return out;
}

} // namespace

// ---------------------------------------------------------------------------
// C ABI
// ---------------------------------------------------------------------------
extern "C" int aaedn_tokenizer_from_bytes(const uint8_t* h_file, size_t n, aaedn_tokenizer** out)
{
    if (!out || (!h_file && n))
        return set_error(AAEDN_EINVAL, "aaedn_tokenizer_from_bytes: null argument");
    *out = nullptr;
    auto* t = new (std::nothrow) aaedn_tokenizer();
    if (!t)
        return set_error(AAEDN_ENOMEM, "aaedn_tokenizer_from_bytes: out of host memory");
    const int rc = parse_abt(h_file, n, *t);
    if (rc)
    {
        delete t;
        return rc;
    }
    *out = t;
    return AAEDN_OK;
}

extern "C" int aaedn_tokenizer_load(const char* path, aaedn_tokenizer** out)
{
    if (!out)
        return set_error(AAEDN_EINVAL, "aaedn_tokenizer_load: null handle pointer");
    *out = nullptr;
    std::vector<uint8_t> img;
    const int rc = read_file(path, img);
    if (rc)
        return rc;
    return aaedn_tokenizer_from_bytes(img.data(), img.size(), out);
}

extern "C" void aaedn_tokenizer_free(aaedn_tokenizer* t) { delete t; }

extern "C" int aaedn_tokenizer_info(const aaedn_tokenizer* t, uint32_t* h_info)
{
    if (!t || !h_info)
        return set_error(AAEDN_EINVAL, "aaedn_tokenizer_info: null argument");
    h_info[0] = t->vocab_size;
    h_info[1] = t->merge_count;
    h_info[2] = t->max_token_bytes;
    h_info[3] = t->format_version;
    h_info[4] = t->payload_checksum;
    return AAEDN_OK;
}

extern "C" int aaedn_tokenizer_encode(const aaedn_tokenizer* t, const char* text, int add_bos, uint32_t* h_ids,
                                      size_t cap, size_t* n_ids)
{
    if (!t || !text || !n_ids || (!h_ids && cap))
        return set_error(AAEDN_EINVAL, "aaedn_tokenizer_encode: null argument");
    std::vector<uint32_t> ids;
    try
    {
        ids = encode_core(t->rule, t->vocab_size, text, add_bos != 0);
    }
    catch (const std::bad_alloc&)
    {
        return set_error(AAEDN_ENOMEM, "aaedn_tokenizer_encode: out of host memory");
    }
    *n_ids = ids.size();
    if (!h_ids)
        return AAEDN_OK; // size query
    if (cap < ids.size())
        return set_error(AAEDN_EINVAL, "aaedn_tokenizer_encode: %zu ids do not fit in %zu", ids.size(), cap);
    std::memcpy(h_ids, ids.data(), ids.size() * 4);
    return AAEDN_OK;
}

extern "C" int aaedn_tokenizer_decode(const aaedn_tokenizer* t, const uint32_t* h_ids, size_t n, char* h_text,
                                      size_t cap, size_t* n_bytes)
{
    if (!t || (!h_ids && n) || !n_bytes || (!h_text && cap))
        return set_error(AAEDN_EINVAL, "aaedn_tokenizer_decode: null argument");
    std::string s;
    try
    {
        s = decode_core(t->strings.data(), t->offsets.data(), t->vocab_size, h_ids, n);
    }
    catch (const std::bad_alloc&)
    {
        return set_error(AAEDN_ENOMEM, "aaedn_tokenizer_decode: out of host memory");
    }
    *n_bytes = s.size();
    if (!h_text)
        return AAEDN_OK; // size query
    if (cap <= s.size())
        return set_error(AAEDN_EINVAL, "aaedn_tokenizer_decode: %zu bytes and a NUL do not fit in %zu", s.size(), cap);
    std::memcpy(h_text, s.data(), s.size());
    h_text[s.size()] = '\0';
    return AAEDN_OK;
}

// ---------------------------------------------------------------------------
// C++ API (the reference's include/tokenizer.hpp): tables in the arena's host
// part; the rule table is rebuilt per encode call (the struct has no slot
// for it).
// ---------------------------------------------------------------------------
namespace aaedn
{

Tokenizer tokenizer_load(Arena* arena, const char* path)
{
    aaedn_tokenizer* h = nullptr;
    if (aaedn_tokenizer_load(path, &h) != AAEDN_OK)
        return Tokenizer{};
    Tokenizer tok{};
    const size_t sb = h->strings.size(); // block + the NUL after it
    char* s = static_cast<char*>(arena_alloc_host(arena, sb, 1));
    auto* off = static_cast<uint32_t*>(arena_alloc_host(arena, (size_t)h->vocab_size * 4, 32));
    auto* f = static_cast<uint16_t*>(arena_alloc_host(arena, (size_t)h->merge_count * 2, 32));
    auto* g = static_cast<uint16_t*>(arena_alloc_host(arena, (size_t)h->merge_count * 2, 32));
    if (!s || (h->vocab_size && !off) || (h->merge_count && (!f || !g)))
    {
        set_error(AAEDN_ENOMEM, "tokenizer_load: the arena's host part cannot hold the tables");
        aaedn_tokenizer_free(h);
        return Tokenizer{};
    }
    std::memcpy(s, h->strings.data(), sb);
    if (h->vocab_size)
        std::memcpy(off, h->offsets.data(), (size_t)h->vocab_size * 4);
    if (h->merge_count)
    {
        std::memcpy(f, h->first.data(), (size_t)h->merge_count * 2);
        std::memcpy(g, h->second.data(), (size_t)h->merge_count * 2);
    }
    tok.strings = s;
    tok.id_to_offset = off;
    tok.merges_first = f;
    tok.merges_second = g;
    tok.vocab_size = h->vocab_size;
    tok.merge_count = h->merge_count;
    tok.max_token_bytes = h->max_token_bytes;
    tok.format_version = h->format_version;
    tok.payload_checksum = h->payload_checksum;
    aaedn_tokenizer_free(h);
    return tok;
}

std::vector<uint32_t> tokenizer_encode(const Tokenizer* tok, const char* text, bool add_bos)
{
    if (!tok || !text)
        return {};
    std::unordered_map<uint32_t, uint32_t> rule;
    if (tok->merge_count && tok->merges_first && tok->merges_second)
        build_rule_table(tok->merges_first, tok->merges_second, tok->merge_count, rule);
    return encode_core(rule, tok->vocab_size, text, add_bos);
}

std::string tokenizer_decode(const Tokenizer* tok, const std::vector<uint32_t>& ids)
{
    if (!tok)
        return {};
    return decode_core(tok->strings, tok->id_to_offset, tok->vocab_size, ids.data(), ids.size());
}

} // namespace aaedn
