// quant_tools.cpp — host-side quant tools of the C ABI (no GPU needed):
// the block quantizer, FNV-1a, the seeded synthetic generator and the RoPE
// tables. Multi-threaded with std::thread; every result is independent of
// the thread count.
#include "aaedn_b200.h"
#include "host_common.hpp"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <thread>
#include <vector>

namespace aaedn_host
{

unsigned worker_count(size_t work_items)
{
    unsigned hw = std::thread::hardware_concurrency();
    if (hw == 0)
        hw = 4;
    hw = std::min(hw, 64u);
    size_t cap = std::max<size_t>(1, work_items / (1u << 16));
    return (unsigned)std::min<size_t>(hw, cap);
}

void parallel_for(size_t n, size_t grain, const std::function<void(size_t, size_t)>& fn)
{
    if (n == 0)
        return;
    unsigned nt = worker_count(n);
    if (nt <= 1)
    {
        fn(0, n);
        return;
    }
    size_t per = (n + nt - 1) / nt;
    per = (per + grain - 1) / grain * grain;
    std::vector<std::thread> th;
    for (size_t b = 0; b < n; b += per)
    {
        size_t e = std::min(n, b + per);
        th.emplace_back([&fn, b, e] { fn(b, e); });
    }
    for (auto& t : th)
        t.join();
}

// binary16 bits from a double, round half to even (what numpy's
// float16(python float) does in tools/convert_model.py:49).
uint16_t f64_to_f16_bits(double d)
{
    uint16_t sign = std::signbit(d) ? 0x8000u : 0u;
    if (std::isnan(d))
        return 0x7E00u;
    double a = std::fabs(d);
    if (a >= 65520.0)
        return sign | 0x7C00u;
    if (a < std::ldexp(1.0, -14))
        return sign | (uint16_t)std::nearbyint(a * std::ldexp(1.0, 24));
    int e = 0;
    double m = std::frexp(a, &e);
    int E = e - 1;
    double r = std::nearbyint(m * 2048.0);
    if (r >= 2048.0)
    {
        r = 1024.0;
        ++E;
    }
    if (E > 15)
        return sign | 0x7C00u;
    return sign | (uint16_t)(((E + 15) << 10) | ((uint32_t)r - 1024u));
}

static inline uint64_t splitmix64(uint64_t x)
{
    uint64_t z = x + 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

static inline uint64_t stream_key(uint64_t seed, uint64_t id)
{
    return splitmix64(seed ^ splitmix64(id + 0x632BE59BD9B4E019ull));
}

// Quantize elements [b, e) of x; b is a multiple of 32.
static void quantize_range(const float* x, size_t n, uint8_t* data, uint16_t* scales, size_t b, size_t e)
{
    for (size_t start = b; start < e; start += 32)
    {
        size_t end = std::min(start + 32, n);
        float mx = 0.0f; // np.max(np.abs(block)) in fp32
        for (size_t i = start; i < end; ++i)
            mx = std::max(mx, std::fabs(x[i]));
        double max_val = (double)mx;
        double scale = max_val > 0.0 ? max_val / 7.0 : 1.0; // fp64 division
        scales[start / 32] = f64_to_f16_bits(scale);
        float sf = (float)scale; // block / scale runs in fp32 (NEP 50)
        for (size_t i = start; i < end; i += 2)
        {
            uint8_t lo = 0, hi = 0;
            if (max_val > 0.0)
            {
                float q0 = std::nearbyint(x[i] / sf);
                lo = (uint8_t)(!(q0 > 0.0f) ? 0 : (q0 > 15.0f ? 15 : (int)q0));
                if (i + 1 < end)
                {
                    float q1 = std::nearbyint(x[i + 1] / sf);
                    hi = (uint8_t)(!(q1 > 0.0f) ? 0 : (q1 > 15.0f ? 15 : (int)q1));
                }
            }
            data[i / 2] = (uint8_t)(lo | (hi << 4));
        }
    }
}

void quantize_q4(const float* x, size_t n, uint8_t* data, uint16_t* scales)
{
    parallel_for(n, 32, [&](size_t b, size_t e) { quantize_range(x, n, data, scales, b, e); });
}

void synth_normal(uint64_t seed, uint64_t id, float std_dev, float* out, size_t n)
{
    const uint64_t key = stream_key(seed, id);
    const double two_pi = 6.283185307179586476925286766559;
    parallel_for(n, 2, [&](size_t b, size_t e) {
        for (size_t i = b; i < e; i += 2)
        {
            uint64_t h = splitmix64(key + (i / 2) * 0x9E3779B97F4A7C15ull);
            double u1 = ((double)(h >> 40) + 1.0) * (1.0 / 16777216.0); // (0, 1]
            double u2 = (double)(h & 0xFFFFFFull) * (1.0 / 16777216.0);  // [0, 1)
            double r = std::sqrt(-2.0 * std::log(u1));
            double t = two_pi * u2;
            out[i] = (float)(std_dev * r * std::cos(t));
            if (i + 1 < e)
                out[i + 1] = (float)(std_dev * r * std::sin(t));
        }
    });
}

void synth_tokens(uint64_t seed, uint64_t id, uint32_t vocab, uint32_t* out, size_t n)
{
    const uint64_t key = stream_key(seed, id ^ 0x746F6B656E73ull);
    for (size_t i = 0; i < n; ++i)
        out[i] = (uint32_t)(splitmix64(key + i * 0x9E3779B97F4A7C15ull) % vocab);
}

} // namespace aaedn_host

using namespace aaedn_host;

extern "C" int aaedn_quantize_q4(const float* h_x, size_t n, uint8_t* h_data, uint16_t* h_scales)
{
    if ((!h_x || !h_data || !h_scales) && n)
        return set_error(AAEDN_EINVAL, "aaedn_quantize_q4: null pointer");
    if (n)
        std::memset(h_data, 0, (n + 1) / 2);
    quantize_q4(h_x, n, h_data, h_scales);
    return AAEDN_OK;
}

extern "C" uint32_t aaedn_fnv1a32(const uint8_t* p, size_t n, uint32_t h)
{
    for (size_t i = 0; i < n; ++i)
    {
        h ^= p[i];
        h *= 0x01000193u;
    }
    return h;
}

extern "C" int aaedn_synth_normal(uint64_t seed, uint64_t tensor_id, float std_dev, float* h_out, size_t n)
{
    if (!h_out && n)
        return set_error(AAEDN_EINVAL, "aaedn_synth_normal: null output");
    synth_normal(seed, tensor_id, std_dev, h_out, n);
    return AAEDN_OK;
}

extern "C" int aaedn_synth_tokens(uint64_t seed, uint64_t stream_id, uint32_t vocab, uint32_t* h_out, size_t n)
{
    if ((!h_out && n) || vocab == 0)
        return set_error(AAEDN_EINVAL, "aaedn_synth_tokens: bad arguments");
    synth_tokens(seed, stream_id, vocab, h_out, n);
    return AAEDN_OK;
}

extern "C" int aaedn_rope_table(float* h_cos, float* h_sin, size_t max_seq, size_t head_dim, double theta,
                                int formula)
{
    if (!h_cos || !h_sin || head_dim < 2 || (head_dim & 1))
        return set_error(AAEDN_EINVAL, "aaedn_rope_table: bad arguments");
    size_t half = head_dim / 2;
    for (size_t pos = 0; pos < max_seq; ++pos)
        for (size_t i = 0; i < half; ++i)
        {
            if (formula == 0)
            {
                // src/rope.cpp:20-29, evaluated in fp32 with the scalar libm
                float freq = 10000.0f / std::pow(2.0f, (float)i / (float)half);
                float angle = (float)pos * freq;
                h_cos[pos * half + i] = std::cos(angle);
                h_sin[pos * half + i] = std::sin(angle);
            }
            else
            {
                double inv = std::pow(theta, -2.0 * (double)i / (double)head_dim);
                double angle = (double)pos * inv;
                h_cos[pos * half + i] = (float)std::cos(angle);
                h_sin[pos * half + i] = (float)std::sin(angle);
            }
        }
    return AAEDN_OK;
}
