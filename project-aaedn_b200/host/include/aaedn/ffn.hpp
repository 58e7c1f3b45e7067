// ffn.hpp — mirror of the reference include/ffn.hpp: what src/ffn.cpp
// computes (the scale of output row j is scales[j/32] as an integer, act =
// g * silu(g) * u), on device pointers, for any ffn_dim (the reference caps
// it at 4096). The model path's SwiGLU (silu(g) * u, fp16 block scales) is
// aaedn_cu_ffn_swiglu(..., AAEDN_FFN_MODEL, ...).
#ifndef AAEDN_B200_FFN_HPP
#define AAEDN_B200_FFN_HPP

#include <cstddef>
#include <cstdint>

namespace aaedn
{

struct QuantBlock;

void ffn_swiglu(const float* input, float* output, size_t batch_size, size_t hidden_dim, size_t ffn_dim,
                const QuantBlock* gate_w, const QuantBlock* up_w, const QuantBlock* down_w, const uint16_t* gate_scales,
                const uint16_t* up_scales, const uint16_t* down_scales);

} // namespace aaedn

#endif
