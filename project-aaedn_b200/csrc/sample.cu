// sample.cu — next-token sampling on the device: temperature, nucleus (top-p)
// filtering and a multinomial draw, the procedure of the reference's sampling
// spec (docs/mpd.md:539-554), without a sort. The draw walks the tokens in the
// spec's sorted order; src/main.cpp:214-247 (softmax, then a draw with
// rand() / RAND_MAX, no temperature or top-p) walks them in id order, which
// samples the same distribution with a different map from u to token.
//
// Order of the vocabulary: probability descending, ties by the lower token id
// (a stable sort). With p_i = exp((l_i - max) / T) (unnormalised, fp32, the
// softmax numerators), Z = sum p_i and the mass of a key k,
// M(k) = sum of p_i over tokens whose key K_i = (bits(p_i) << 32 | ~i) >= k
// (the cumulative sum up to and including the token with key k in that
// order), the nucleus ends at the first token whose cumulative sum reaches
// top_p * Z, i.e. at k_top = max{K_i : M(K_i) >= top_p * Z}; with kept mass
// W = M(k_top), the draw is the first token whose cumulative sum reaches
// u * W: max{K_i : M(K_i) >= u * W} (u in [0, 1), so it lies in the nucleus).
// Both are found by a radix select over the 64-bit keys, 8 bits a pass, on
// masses summed in fp64. T <= 0 is greedy: the argmax, ties to the lowest id.
#include "common.cuh"

#include "aaedn_b200.h"
#include "host_common.hpp"

using namespace aaedn_dev;

namespace
{

constexpr int SAMPLE_THREADS = 1024;
constexpr int SAMPLE_WARPS = SAMPLE_THREADS / 32;
constexpr int SAMPLE_BINS = 256;

__device__ __forceinline__ uint64_t sample_key(float p, uint32_t i)
{
    return ((uint64_t)__float_as_uint(p) << 32) | (uint64_t)(0xFFFFFFFFu - i);
}

// Block-wide fp64 sum (every thread gets it); red: SAMPLE_WARPS doubles.
__device__ double block_sum_f64(double v, double* red)
{
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
        v += __shfl_xor_sync(0xffffffffu, v, o);
    __syncthreads();
    if (lane == 0)
        red[warp] = v;
    __syncthreads();
    double t = 0.0;
    for (int w = 0; w < SAMPLE_WARPS; ++w) // fixed order
        t += red[w];
    return t;
}

// max{K_i : M(K_i) >= target} over the vocabulary, and M of that key in
// *mass_out (the same value in every thread).
// hist: SAMPLE_WARPS x SAMPLE_BINS doubles of shared memory; tot: SAMPLE_BINS.
__device__ uint64_t select_key(const float* __restrict__ logits, uint32_t V, float mx, float inv_t, double target,
                               double* hist, double* tot, double* mass_out)
{
    const int tid = threadIdx.x, warp = tid >> 5;
    uint64_t prefix = 0;   // the key's bits chosen so far
    double above = 0.0;    // mass of the keys above the current prefix range
    for (int level = 7; level >= 0; --level)
    {
        const int shift = level * 8;
        for (int i = tid; i < SAMPLE_WARPS * SAMPLE_BINS; i += SAMPLE_THREADS)
            hist[i] = 0.0;
        __syncthreads();
        double* mine = hist + warp * SAMPLE_BINS;
        for (uint32_t i = tid; i < V; i += SAMPLE_THREADS)
        {
            const float p = expf((logits[i] - mx) * inv_t);
            const uint64_t k = sample_key(p, i);
            // candidates: keys that agree with the prefix above this level
            const bool cand = level == 7 || (k >> (shift + 8)) == (prefix >> (shift + 8));
            if (cand && p > 0.0f)
                atomicAdd(mine + ((k >> shift) & 0xFF), (double)p);
        }
        __syncthreads();
        for (int b = tid; b < SAMPLE_BINS; b += SAMPLE_THREADS)
        {
            double s = 0.0;
            for (int w = 0; w < SAMPLE_WARPS; ++w)
                s += hist[w * SAMPLE_BINS + b];
            tot[b] = s;
        }
        __syncthreads();
        // the largest bin b with above + sum(tot[b..255]) >= target (bins of
        // zero mass are skipped: the chosen one holds a token)
        double acc = above;
        int pick = -1;
        for (int b = SAMPLE_BINS - 1; b >= 0; --b)
        {
            if (tot[b] <= 0.0)
                continue;
            if (acc + tot[b] >= target)
            {
                pick = b;
                break;
            }
            acc += tot[b];
        }
        if (pick < 0) // rounding left target above the whole mass: take the last token
        {
            for (int b = 0; b < SAMPLE_BINS; ++b)
                if (tot[b] > 0.0)
                {
                    pick = b;
                    break;
                }
            acc = above;
            for (int b = SAMPLE_BINS - 1; b > pick; --b)
                acc += tot[b];
            if (pick < 0)
                pick = 0;
        }
        above = acc;
        prefix |= (uint64_t)pick << shift;
        __syncthreads(); // tot is rewritten by the next level
    }
    // the key is now exact: one token; M(key) = above + its p
    *mass_out = above + (double)__uint_as_float((uint32_t)(prefix >> 32));
    return prefix;
}

__global__ void __launch_bounds__(SAMPLE_THREADS, 1)
    sample_kernel(const float* __restrict__ logits, uint32_t V, float temperature, float top_p, float u,
                  uint32_t* __restrict__ out)
{
    extern __shared__ __align__(16) double ssm[];
    double* hist = ssm;                                   // SAMPLE_WARPS x SAMPLE_BINS
    double* tot = hist + SAMPLE_WARPS * SAMPLE_BINS;      // SAMPLE_BINS
    double* red = tot + SAMPLE_BINS;                      // SAMPLE_WARPS
    __shared__ float s_v[SAMPLE_WARPS];
    __shared__ uint32_t s_i[SAMPLE_WARPS];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

    // argmax, ties to the lowest id (also the max of the softmax)
    float bv = -INFINITY;
    uint32_t bi = 0xFFFFFFFFu;
    for (uint32_t i = tid; i < V; i += SAMPLE_THREADS)
    {
        const float v = logits[i];
        if (v > bv || (v == bv && i < bi))
        {
            bv = v;
            bi = i;
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
    {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const uint32_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > bv || (ov == bv && oi < bi))
        {
            bv = ov;
            bi = oi;
        }
    }
    if (lane == 0)
    {
        s_v[warp] = bv;
        s_i[warp] = bi;
    }
    __syncthreads();
    bv = s_v[0];
    bi = s_i[0];
    for (int w = 1; w < SAMPLE_WARPS; ++w)
        if (s_v[w] > bv || (s_v[w] == bv && s_i[w] < bi))
        {
            bv = s_v[w];
            bi = s_i[w];
        }
    if (!(temperature > 0.0f) || !(bv > -INFINITY) || !isfinite(bv))
    {
        // greedy (T <= 0), or no finite logit to normalise by
        if (tid == 0)
            *out = bi == 0xFFFFFFFFu ? 0u : bi;
        return;
    }
    // (l - max) / T as (l - max) * (1 / T): the spec divides the logits by T
    // before the softmax's max subtraction; this order keeps T = 1 bit-exact
    // with src/main.cpp:226 (expf(logits[i] - max_val))
    const float inv_t = 1.0f / temperature;
    const float mx = bv;
    double z = 0.0;
    for (uint32_t i = tid; i < V; i += SAMPLE_THREADS)
        z += (double)expf((logits[i] - mx) * inv_t);
    z = block_sum_f64(z, red);
    double w_top = 0.0, w_draw = 0.0;
    select_key(logits, V, mx, inv_t, (double)top_p * z, hist, tot, &w_top);
    const uint64_t k = select_key(logits, V, mx, inv_t, (double)u * w_top, hist, tot, &w_draw);
    if (tid == 0)
        *out = 0xFFFFFFFFu - (uint32_t)(k & 0xFFFFFFFFu);
}

int check_device_ptr(const void* p, const char* what)
{
    if (!p)
        return set_error(AAEDN_EINVAL, "%s is null", what);
    cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess)
    {
        cudaGetLastError();
        return set_error(AAEDN_EINVAL, "%s: cannot query pointer", what);
    }
    if (a.type != cudaMemoryTypeDevice && a.type != cudaMemoryTypeManaged)
        return set_error(AAEDN_EINVAL, "%s is not device memory", what);
    return AAEDN_OK;
}

} // namespace

extern "C" int aaedn_cu_sample(const float* d_logits, uint32_t vocab, float temperature, float top_p, float u,
                               uint32_t* d_token, void* stream)
{
    if (vocab == 0 || vocab > 0x7FFFFFFFu)
        return set_error(AAEDN_EINVAL, "aaedn_cu_sample: vocab %u", vocab);
    if (!(top_p > 0.0f && top_p <= 1.0f))
        return set_error(AAEDN_EINVAL, "aaedn_cu_sample: top_p %g outside (0, 1]", (double)top_p);
    if (!(u >= 0.0f && u < 1.0f))
        return set_error(AAEDN_EINVAL, "aaedn_cu_sample: u %g outside [0, 1)", (double)u);
    if (int rc = check_device_ptr(d_logits, "d_logits"))
        return rc;
    if (int rc = check_device_ptr(d_token, "d_token"))
        return rc;
    const size_t smem = ((size_t)SAMPLE_WARPS * SAMPLE_BINS + SAMPLE_BINS + SAMPLE_WARPS) * sizeof(double);
    AAEDN_CUDA_TRY(cudaFuncSetAttribute(sample_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    sample_kernel<<<1, SAMPLE_THREADS, smem, as_stream(stream)>>>(d_logits, vocab, temperature, top_p, u, d_token);
    AAEDN_LAUNCH_CHECK("sample_kernel");
    return AAEDN_OK;
}
