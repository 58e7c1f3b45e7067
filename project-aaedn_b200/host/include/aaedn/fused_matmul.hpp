// fused_matmul.hpp — mirror of the reference include/fused_matmul.hpp.
// output[m*ldc+n] = sum_k input[m*lda+k] * code(n,k) * scale(n,k/32) with
// weights [N][K] (ldb codes per row) and fp16 block scales; device pointers,
// asynchronous on the legacy default stream. init/destroy keep no state (the
// kernel needs no scratch).
#ifndef AAEDN_B200_FUSED_MATMUL_HPP
#define AAEDN_B200_FUSED_MATMUL_HPP

#include <cstddef>
#include <cstdint>

namespace aaedn
{

struct Arena;

void fused_matmul_init(Arena* arena);
void fused_matmul(const float* input, const uint8_t* weights, const uint16_t* scales, float* output, size_t M, size_t N,
                  size_t K, size_t lda, size_t ldb, size_t ldc);
void fused_matmul_destroy();

} // namespace aaedn

#endif
