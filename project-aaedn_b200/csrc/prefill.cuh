// prefill.cuh — the token loop over many prompt tokens at once
// (src/transformer.cpp:128-243 with decision D7: every input token is
// processed, from the sequence's position on). The matrix products are the
// tcgen05 GEMM (gemm_tc.cuh) with the model's epilogues; around them:
//   * pf_embed_kernel: the residual rows of the chunk's tokens (:144-146);
//   * pf_rmsnorm_split_kernel: RMSNorm of each residual row (:150-153,
//     :217-220; src/rmsnorm.cpp:8-51) written straight as the GEMM's three
//     bf16 activation parts;
//   * attn_prefill_kernel: causal attention of each chunk token over the
//     cache up to its own position (D4), after the QKV epilogue appended the
//     chunk's K/V rows.
#pragma once

#include "common.cuh"
#include "gemv_q4.cuh" // block_sum

namespace aaedn_dev
{

// hidden[t][:] = embedding[tokens[t]][:] for t < n
__global__ void pf_embed_kernel(const uint32_t* __restrict__ tokens, int n, const float* __restrict__ embedding, int D,
                                float* __restrict__ hidden)
{
    const int t = blockIdx.x;
    if (t >= n)
        return;
    const float4* src = reinterpret_cast<const float4*>(embedding + (size_t)tokens[t] * D);
    float4* dst = reinterpret_cast<float4*>(hidden + (size_t)t * D);
    for (int i = threadIdx.x; i < D / 4; i += blockDim.x)
        dst[i] = src[i];
}

// One CTA per row m < M_pad: parts[q][m][k] (q = 0, 1, 2: the bf16 parts of
// x * rms * g, src/rmsnorm.cpp:34-43); rows m >= M are zero.
__global__ void __launch_bounds__(256) pf_rmsnorm_split_kernel(const float* __restrict__ x, int D, int M, int M_pad,
                                                               const float* __restrict__ gain, float eps,
                                                               __nv_bfloat16* __restrict__ parts)
{
    __shared__ float scratch[64];
    const int m = blockIdx.x;
    const size_t plane = (size_t)M_pad * D;
    __nv_bfloat16* p0 = parts + (size_t)m * D;
    if (m >= M)
    {
        for (int k = threadIdx.x; k < D; k += blockDim.x)
            p0[k] = p0[k + plane] = p0[k + 2 * plane] = __float2bfloat16_rn(0.0f);
        return;
    }
    const float* xr = x + (size_t)m * D;
    float ss = 0.0f;
    for (int k = threadIdx.x; k < D; k += blockDim.x)
        ss = fmaf(xr[k], xr[k], ss);
    ss = block_sum(ss, scratch);
    const float rms = 1.0f / sqrtf(__fadd_rn(__fdiv_rn(ss, (float)D), eps));
    for (int k = threadIdx.x; k < D; k += blockDim.x)
    {
        const float v = __fmul_rn(__fmul_rn(xr[k], rms), gain[k]);
        const __nv_bfloat16 h = __float2bfloat16_rn(v);
        const float r1 = v - __bfloat162float(h);
        const __nv_bfloat16 md = __float2bfloat16_rn(r1);
        p0[k] = h;
        p0[k + plane] = md;
        p0[k + 2 * plane] = __float2bfloat16_rn(r1 - __bfloat162float(md));
    }
}

constexpr int PF_ATTN_WARPS = 4;

// Causal attention of chunk tokens t < n (positions pos0 + t) for query head
// blockIdx.x: one warp per token. Keys are taken 32 at a time, lane j scoring
// key s0 + j against q (held in shared memory); the batch's softmax weights
// then scale the V rows with lanes over the head dims; the softmax is carried
// online across batches (running max and sum). fp32, expf (D4).
// out[t][h * hd + d]; head_dim a multiple of 32, <= 256.
__global__ void __launch_bounds__(PF_ATTN_WARPS * 32) attn_prefill_kernel(
    const float* __restrict__ q, size_t ldq, const float* __restrict__ k_layer, const float* __restrict__ v_layer,
    const int* __restrict__ page_table, int page_size, int n_heads, int n_kv, int hd, int pos0, int n, float scale,
    float* __restrict__ out, size_t ldo)
{
    __shared__ __align__(16) float qs[PF_ATTN_WARPS][256];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int h = blockIdx.x, t = blockIdx.y * PF_ATTN_WARPS + warp;
    if (t >= n)
        return;
    const int kvh = h / (n_heads / n_kv);
    const int pos = pos0 + t, nkeys = pos + 1;
    const float* qh = q + (size_t)t * ldq + (size_t)h * hd;
    for (int d = lane; d < hd; d += 32)
        qs[warp][d] = qh[d];
    __syncwarp();
    const int dpl = hd >> 5; // dims per lane in the V accumulation
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    float mrun = -INFINITY, lrun = 0.0f;
    for (int s0 = 0; s0 < nkeys; s0 += 32)
    {
        const int s = s0 + lane;
        float sc = -INFINITY;
        if (s < nkeys)
        {
            const int page = page_table[s / page_size];
            const float4* kr = reinterpret_cast<const float4*>(
                k_layer + (((size_t)page * n_kv + kvh) * page_size + (s % page_size)) * hd);
            const float4* q4 = reinterpret_cast<const float4*>(qs[warp]);
            float dot = 0.0f;
            for (int c = 0; c < (hd >> 2); ++c)
            {
                const float4 kv = kr[c], qv = q4[c];
                dot = fmaf(qv.x, kv.x, dot);
                dot = fmaf(qv.y, kv.y, dot);
                dot = fmaf(qv.z, kv.z, dot);
                dot = fmaf(qv.w, kv.w, dot);
            }
            sc = dot * scale; // src/attention.cpp:36-41
        }
        const float bmax = warp_max(sc);
        const float mnew = fmaxf(mrun, bmax);
        const float w = (s < nkeys) ? expf(sc - mnew) : 0.0f;
        const float corr = (mrun == -INFINITY) ? 0.0f : expf(mrun - mnew);
        lrun = lrun * corr + warp_sum(w);
        mrun = mnew;
#pragma unroll
        for (int i = 0; i < 8; ++i)
            acc[i] *= corr;
        const int nb = min(32, nkeys - s0);
        for (int j = 0; j < nb; ++j)
        {
            const float wj = __shfl_sync(0xffffffffu, w, j);
            const int sj = s0 + j;
            const int page = page_table[sj / page_size];
            const float* vr = v_layer + (((size_t)page * n_kv + kvh) * page_size + (sj % page_size)) * hd;
#pragma unroll
            for (int i = 0; i < 8; ++i)
                if (i < dpl)
                    acc[i] = fmaf(wj, vr[lane + 32 * i], acc[i]);
        }
    }
    const float inv = 1.0f / lrun;
    float* o = out + (size_t)t * ldo + (size_t)h * hd;
#pragma unroll
    for (int i = 0; i < 8; ++i)
        if (i < dpl)
            o[lane + 32 * i] = acc[i] * inv;
}

} // namespace aaedn_dev
