// host_common.hpp — shared host-side helpers of libaaedn_b200 (error state,
// thread pool helpers, fp16 conversion, synthetic generator).
#ifndef AAEDN_HOST_COMMON_HPP
#define AAEDN_HOST_COMMON_HPP

#include <cstddef>
#include <cstdint>
#include <functional>

namespace aaedn_host
{

// Records msg as the calling thread's last error and returns code.
int set_error(int code, const char* fmt, ...);

unsigned worker_count(size_t work_items);
void parallel_for(size_t n, size_t grain, const std::function<void(size_t, size_t)>& fn);

uint16_t f64_to_f16_bits(double d);
void quantize_q4(const float* x, size_t n, uint8_t* data, uint16_t* scales);
void synth_normal(uint64_t seed, uint64_t id, float std_dev, float* out, size_t n);
void synth_tokens(uint64_t seed, uint64_t id, uint32_t vocab, uint32_t* out, size_t n);

} // namespace aaedn_host

#endif
