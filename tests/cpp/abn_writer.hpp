// Test helper: writes .abn v2 files the way tools/convert_model.py:130-150
// does ("<8sIQI6IB15s" header, then codes and u16 scales, FNV-1a checksum).
#pragma once
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

namespace abn_test
{

inline uint32_t fnv1a(const uint8_t* p, size_t n, uint32_t h = 0x811C9DC5u)
{
    for (size_t i = 0; i < n; ++i)
    {
        h ^= p[i];
        h *= 0x01000193u;
    }
    return h;
}

struct Dims
{
    uint32_t n_layers = 2, n_heads = 4, head_dim = 32, vocab = 1000, hidden = 128, ffn = 256;
};

inline std::vector<uint8_t> header(uint32_t version, uint64_t payload_size, uint32_t checksum, const Dims& d,
                                   const char* magic = "AAEDNMDL")
{
    std::vector<uint8_t> out(magic, magic + 8);
    auto u32 = [&](uint32_t v) {
        for (int i = 0; i < 4; ++i)
            out.push_back((uint8_t)(v >> (8 * i)));
    };
    u32(version);
    for (int i = 0; i < 8; ++i)
        out.push_back((uint8_t)(payload_size >> (8 * i)));
    u32(checksum);
    u32(d.n_layers);
    u32(d.n_heads);
    u32(d.head_dim);
    u32(d.vocab);
    u32(d.hidden);
    u32(d.ffn);
    out.push_back(0);
    out.insert(out.end(), 15, 0);
    return out;
}

// A valid file: hidden x hidden codes (deterministic pattern) and scales.
inline std::vector<uint8_t> valid_model(const Dims& d, std::vector<uint8_t>* codes_out = nullptr,
                                        std::vector<uint16_t>* scales_out = nullptr)
{
    const size_t h = d.hidden;
    std::vector<uint8_t> codes(h * h / 2);
    std::vector<uint16_t> scales(h * h / 32);
    for (size_t i = 0; i < codes.size(); ++i)
        codes[i] = (uint8_t)((i * 37 + 11) & 0xFF);
    for (size_t i = 0; i < scales.size(); ++i)
        scales[i] = (uint16_t)(0x2000 + (i * 7) % 0x1000);
    std::vector<uint8_t> payload(codes.begin(), codes.end());
    const uint8_t* sp = reinterpret_cast<const uint8_t*>(scales.data());
    payload.insert(payload.end(), sp, sp + scales.size() * 2);
    auto out = header(2, payload.size(), fnv1a(payload.data(), payload.size()), d);
    out.insert(out.end(), payload.begin(), payload.end());
    if (codes_out)
        *codes_out = codes;
    if (scales_out)
        *scales_out = scales;
    return out;
}

// A whole-model file (the layout aaedn_abn_model_read_header documents):
// version 3, n_kv_heads / rope_theta / eps in the reserved bytes, then the
// given payload.
inline std::vector<uint8_t> whole_model_header(const Dims& d, uint32_t n_kv_heads, float theta, float eps,
                                               const std::vector<uint8_t>& payload)
{
    std::vector<uint8_t> out = header(3, payload.size(), fnv1a(payload.data(), payload.size()), d);
    auto put = [&](size_t at, const void* v) { std::memcpy(out.data() + at, v, 4); };
    put(49, &n_kv_heads);
    put(53, &theta);
    put(57, &eps);
    return out;
}

template <typename T>
inline void append(std::vector<uint8_t>& out, const std::vector<T>& v)
{
    const uint8_t* p = reinterpret_cast<const uint8_t*>(v.data());
    out.insert(out.end(), p, p + v.size() * sizeof(T));
}

inline void write_file(const std::string& path, const std::vector<uint8_t>& data)
{
    FILE* f = std::fopen(path.c_str(), "wb");
    std::fwrite(data.data(), 1, data.size(), f);
    std::fclose(f);
}

} // namespace abn_test
