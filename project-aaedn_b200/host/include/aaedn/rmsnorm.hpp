// rmsnorm.hpp — mirror of the reference include/rmsnorm.hpp (device
// pointers, asynchronous on the legacy default stream).
#ifndef AAEDN_B200_RMSNORM_HPP
#define AAEDN_B200_RMSNORM_HPP

#include <cstddef>
#include <cstdint>

namespace aaedn
{

void rmsnorm(const float* input, float* output, const float* weight, size_t n, float eps = 1e-6f);

}

#endif
