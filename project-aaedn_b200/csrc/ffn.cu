// ffn.cu — the standalone SwiGLU FFN entry point (include/ffn.hpp:12,
// src/ffn.cpp:18-77) and the device-to-device copy used by the C++ KV-cache
// API.
//
// Two semantics:
//  * AAEDN_FFN_MODEL: the model path's FFN (decisions D1/D2/D6): fp16 block
//    scales per (row, 32 inputs), act = silu(g) * u. Built from the
//    dequant-GEMV (aaedn_cu_fused_matmul) and one elementwise kernel.
//  * AAEDN_FFN_REFERENCE: what src/ffn.cpp computes, for drop-in parity: the
//    u16 scale of output row j is scales[j / 32] cast as an integer
//    (src/ffn.cpp:41,52,72), act = g * silu(g) * u (src/ffn.cpp:62,72).
//    A warp per output row; this is an API-parity path, not the decode path.
#include "common.cuh"

#include "aaedn_b200.h"
#include "host_common.hpp"

using namespace aaedn_dev;

namespace
{

// out[b][j] = sum_i in[b][i] * code(j, i) * (float)scales[j / 32]
__global__ void rowscale_gemv_kernel(const float* __restrict__ in, const uint8_t* __restrict__ w,
                                     const uint16_t* __restrict__ scales, float* __restrict__ out, int B, int N, int K)
{
    const int warps = blockDim.x >> 5, lane = threadIdx.x & 31;
    const int j = blockIdx.x * warps + (threadIdx.x >> 5);
    if (j >= N)
        return;
    const uint8_t* row = w + (size_t)j * (K / 2);
    const float s = (float)scales[j / 32];
    for (int b = 0; b < B; ++b)
    {
        const float* x = in + (size_t)b * K;
        float acc = 0.0f;
        for (int i = lane; i < K; i += 32)
        {
            const int code = (row[i >> 1] >> ((i & 1) * 4)) & 0x0F;
            acc = fmaf(x[i], (float)code * s, acc);
        }
        acc = warp_sum(acc);
        if (lane == 0)
            out[(size_t)b * N + j] = acc;
    }
}

// act = silu(g) * u (model) or g * silu(g) * u (reference), in place into g
__global__ void swiglu_kernel(float* __restrict__ g, const float* __restrict__ u, size_t n, int reference)
{
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n)
        return;
    const float gv = g[i];
    g[i] = reference ? __fmul_rn(__fmul_rn(gv, silu_f(gv)), u[i]) : __fmul_rn(silu_f(gv), u[i]);
}

} // namespace

extern "C" int aaedn_memcpy_d2d(void* d_dst, const void* d_src, size_t bytes, void* stream)
{
    AAEDN_CUDA_TRY(cudaMemcpyAsync(d_dst, d_src, bytes, cudaMemcpyDeviceToDevice,
                                   static_cast<cudaStream_t>(stream)));
    return AAEDN_OK;
}

extern "C" int aaedn_cu_ffn_swiglu(const float* d_in, float* d_out, size_t batch, size_t hidden, size_t ffn,
                                   const uint8_t* d_gate, const uint8_t* d_up, const uint8_t* d_down,
                                   const uint16_t* d_gate_scales, const uint16_t* d_up_scales,
                                   const uint16_t* d_down_scales, int semantics, void* stream)
{
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (batch == 0 || hidden == 0)
        return AAEDN_OK;
    if (!d_out)
        return set_error(AAEDN_EINVAL, "aaedn_cu_ffn_swiglu: null output");
    if (!d_in || !d_gate || !d_up || !d_down || !d_gate_scales || !d_up_scales || !d_down_scales || ffn == 0)
    {
        // src/ffn.cpp:22-27 writes zeros (of the first row; all rows here)
        AAEDN_CUDA_TRY(cudaMemsetAsync(d_out, 0, batch * hidden * sizeof(float), st));
        return AAEDN_OK;
    }
    if (semantics != AAEDN_FFN_MODEL && semantics != AAEDN_FFN_REFERENCE)
        return set_error(AAEDN_EINVAL, "aaedn_cu_ffn_swiglu: semantics %d", semantics);
    if (hidden % 32 || ffn % 32 || batch > 65535 || hidden > (1u << 24) || ffn > (1u << 24))
        return set_error(AAEDN_EINVAL, "aaedn_cu_ffn_swiglu: hidden and ffn must be multiples of 32");
    float* g = nullptr;
    AAEDN_CUDA_TRY(cudaMallocAsync(reinterpret_cast<void**>(&g), 2 * batch * ffn * sizeof(float), st));
    float* u = g + batch * ffn;
    int rc = AAEDN_OK;
    if (semantics == AAEDN_FFN_MODEL)
    {
        rc = aaedn_cu_fused_matmul(d_in, d_gate, d_gate_scales, g, batch, ffn, hidden, hidden, hidden, ffn,
                                   AAEDN_SCALE_F16, stream);
        if (!rc)
            rc = aaedn_cu_fused_matmul(d_in, d_up, d_up_scales, u, batch, ffn, hidden, hidden, hidden, ffn,
                                       AAEDN_SCALE_F16, stream);
    }
    else
    {
        const unsigned blocks = (unsigned)((ffn + 7) / 8);
        rowscale_gemv_kernel<<<blocks, 256, 0, st>>>(d_in, d_gate, d_gate_scales, g, (int)batch, (int)ffn,
                                                     (int)hidden);
        cudaError_t e = cudaGetLastError();
        if (e == cudaSuccess)
        {
            count_launch();
            rowscale_gemv_kernel<<<blocks, 256, 0, st>>>(d_in, d_up, d_up_scales, u, (int)batch, (int)ffn,
                                                         (int)hidden);
            e = cudaGetLastError();
            count_launch();
        }
        if (e != cudaSuccess)
            rc = set_error(AAEDN_ECUDA, "aaedn_cu_ffn_swiglu: %s", cudaGetErrorString(e));
    }
    if (!rc)
    {
        const size_t n = batch * ffn;
        swiglu_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(g, u, n, semantics == AAEDN_FFN_REFERENCE);
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess)
            rc = set_error(AAEDN_ECUDA, "aaedn_cu_ffn_swiglu: %s", cudaGetErrorString(e));
        else
            count_launch();
    }
    if (!rc)
    {
        if (semantics == AAEDN_FFN_MODEL)
            rc = aaedn_cu_fused_matmul(g, d_down, d_down_scales, d_out, batch, hidden, ffn, ffn, ffn, hidden,
                                       AAEDN_SCALE_F16, stream);
        else
        {
            rowscale_gemv_kernel<<<(unsigned)((hidden + 7) / 8), 256, 0, st>>>(g, d_down, d_down_scales, d_out,
                                                                               (int)batch, (int)hidden, (int)ffn);
            cudaError_t e = cudaGetLastError();
            if (e != cudaSuccess)
                rc = set_error(AAEDN_ECUDA, "aaedn_cu_ffn_swiglu: %s", cudaGetErrorString(e));
            else
                count_launch();
        }
    }
    cudaError_t fe = cudaFreeAsync(g, st);
    if (!rc && fe != cudaSuccess)
        rc = set_error(AAEDN_ECUDA, "aaedn_cu_ffn_swiglu: %s", cudaGetErrorString(fe));
    return rc;
}
