// attention.cuh — split-K decode attention (one query token per head) over
// either a segment list (the reference API, src/attention.cpp:10-84) or a
// paged KV cache (the model path, D4/D5: causal MHA/GQA at the token's
// position).
//
// Grid (n_kv_heads, S): CTA (h, s) owns tokens [L*s/S, L*(s+1)/S) of kv head
// h and all G = n_heads/n_kv query heads that share it, so each K/V row is
// read from HBM once per step. Inside a CTA the scores are exact (max, then
// exp(s - max), then the V sum: the three passes of src/attention.cpp:46-82);
// the S partial results (max, sum, unnormalised output) are merged by the
// last CTA of each kv head in fixed split order, so the result is
// deterministic. All arithmetic is fp32 with expf.
#pragma once

#include "gemv_q4.cuh"

namespace aaedn_dev
{

constexpr int ATTN_THREADS = 128;
constexpr int ATTN_MAX_SEG = 64;
constexpr int ATTN_MAX_HD = 256;

struct AttnParams
{
    const float* q; // [n_heads][hd]
    const float* k; // MODE 0: [token][n_heads][hd]; MODE 1: [page][n_kv][P][hd]
    const float* v;
    float* out;         // [n_heads][hd]
    float* part;        // [n_heads][S][hd + 2]
    unsigned* counters; // [n_kv], zero between launches
    int n_heads, n_kv, head_dim, S;
    float scale;
    const DecodeState* state; // MODE 1: L = pos + 1
    int len_static;           // MODE 0: L
    int max_len;              // bound on L (cache capacity)
    int max_tok;              // smem bound on tokens per split
    const int* page_table;
    int page_size;
    int nseg;
    uint32_t seg_start[ATTN_MAX_SEG];
    uint32_t seg_off[ATTN_MAX_SEG + 1]; // prefix sums of the lengths
};

inline size_t attn_smem_bytes(int G, int hd, int max_tok)
{
    return ((size_t)G * hd + (size_t)G * max_tok + (size_t)G * hd * (ATTN_THREADS / 16) + 64) * 4;
}

template <int MODE>
__device__ __forceinline__ size_t attn_row(const AttnParams& p, int t, int kvh)
{
    const int hd = p.head_dim;
    if constexpr (MODE == 0)
    {
        int j = 0;
        while (j + 1 < p.nseg && (uint32_t)t >= p.seg_off[j + 1])
            ++j;
        const uint32_t phys = p.seg_start[j] + ((uint32_t)t - p.seg_off[j]);
        return ((size_t)phys * p.n_heads + kvh) * hd;
    }
    else
    {
        const int page = p.page_table[t / p.page_size];
        return (((size_t)page * p.n_kv + kvh) * p.page_size + (t % p.page_size)) * hd;
    }
}

template <int MODE>
__global__ void __launch_bounds__(ATTN_THREADS) attn_split_kernel(const AttnParams p)
{
    extern __shared__ __align__(16) float asmem[];
    const int kvh = blockIdx.x, split = blockIdx.y, S = p.S;
    const int G = p.n_heads / p.n_kv, hd = p.head_dim;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    int L = (MODE == 1) ? (int)p.state->pos + 1 : p.len_static;
    if (L > p.max_len)
        L = p.max_len;
    const int t0 = (int)(((long long)L * split) / S);
    const int t1 = (int)(((long long)L * (split + 1)) / S);
    const int ntok = t1 - t0;

    float* qs = asmem;                  // [G][hd]
    float* sc = qs + G * hd;            // [G][max_tok]
    float* ored = sc + G * p.max_tok;   // [ATTN_THREADS/16][G][hd] partial V sums
    float* misc = ored + (ATTN_THREADS / 16) * G * hd; // 64

    for (int i = tid; i < G * hd; i += ATTN_THREADS)
        qs[i] = p.q[(size_t)kvh * G * hd + i];
    __syncthreads();

    // pass 1: scores (one warp per token, lanes over the head dimension)
    constexpr int ND = ATTN_MAX_HD / 32;
    for (int j = warp; j < ntok; j += ATTN_THREADS / 32)
    {
        const float* kr = p.k + attn_row<MODE>(p, t0 + j, kvh);
        float kv[ND];
#pragma unroll
        for (int c = 0; c < ND; ++c)
        {
            const int d = lane + 32 * c;
            kv[c] = d < hd ? kr[d] : 0.0f;
        }
        for (int gi = 0; gi < G; ++gi)
        {
            float dot = 0.0f;
#pragma unroll
            for (int c = 0; c < ND; ++c)
            {
                const int d = lane + 32 * c;
                if (d < hd)
                    dot = fmaf(qs[gi * hd + d], kv[c], dot);
            }
            dot = warp_sum(dot);
            if (lane == 0)
                sc[gi * p.max_tok + j] = dot * p.scale; // src/attention.cpp:42
        }
    }
    __syncthreads();

    // pass 2: max and exp per query head (src/attention.cpp:46-59)
    for (int gi = warp; gi < G; gi += ATTN_THREADS / 32)
    {
        float mx = -INFINITY;
        for (int j = lane; j < ntok; j += 32)
            mx = fmaxf(mx, sc[gi * p.max_tok + j]);
        mx = warp_max(mx);
        float sum = 0.0f;
        for (int j = lane; j < ntok; j += 32)
        {
            const float e = expf(sc[gi * p.max_tok + j] - mx);
            sc[gi * p.max_tok + j] = e;
            sum += e;
        }
        sum = warp_sum(sum);
        if (lane == 0)
        {
            misc[2 * gi] = mx;
            misc[2 * gi + 1] = sum;
        }
    }
    __syncthreads();

    // pass 3: unnormalised sum of e * v; thread = (token lane j0, dim d)
    {
        const int nsub = ATTN_THREADS / 16; // 8 token lanes
        const int dl = tid & 15, j0 = tid >> 4;
        for (int gi = 0; gi < G; ++gi)
            for (int d = dl; d < hd; d += 16)
                ored[(j0 * G + gi) * hd + d] = 0.0f;
        for (int j = j0; j < ntok; j += nsub)
        {
            const float* vr = p.v + attn_row<MODE>(p, t0 + j, kvh);
            for (int d = dl; d < hd; d += 16)
            {
                const float vv = vr[d];
                for (int gi = 0; gi < G; ++gi)
                    ored[(j0 * G + gi) * hd + d] = fmaf(sc[gi * p.max_tok + j], vv, ored[(j0 * G + gi) * hd + d]);
            }
        }
    }
    __syncthreads();
    for (int i = tid; i < G * hd; i += ATTN_THREADS)
    {
        const int gi = i / hd, d = i - gi * hd;
        float o = 0.0f;
        for (int j0 = 0; j0 < ATTN_THREADS / 16; ++j0)
            o += ored[(j0 * G + gi) * hd + d];
        const int h = kvh * G + gi;
        float* pp = p.part + ((size_t)h * S + split) * (hd + 2);
        pp[d] = o;
        if (d == 0)
        {
            pp[hd] = misc[2 * gi];
            pp[hd + 1] = misc[2 * gi + 1];
        }
    }

    // last CTA of this kv head merges the S splits in order
    __threadfence();
    __syncthreads();
    __shared__ unsigned s_last;
    if (tid == 0)
    {
        const unsigned prev = atomicAdd(&p.counters[kvh], 1u);
        s_last = (prev == (unsigned)S - 1) ? 1u : 0u;
    }
    __syncthreads();
    if (!s_last)
        return;
    __threadfence();
    for (int i = tid; i < G * hd; i += ATTN_THREADS)
    {
        const int gi = i / hd, d = i - gi * hd;
        const int h = kvh * G + gi;
        const float* pb = p.part + (size_t)h * S * (hd + 2);
        float M = -INFINITY;
        for (int s2 = 0; s2 < S; ++s2)
            M = fmaxf(M, __ldcg(pb + (size_t)s2 * (hd + 2) + hd));
        float num = 0.0f, den = 0.0f;
        for (int s2 = 0; s2 < S; ++s2)
        {
            const float ms = __ldcg(pb + (size_t)s2 * (hd + 2) + hd);
            const float w = (ms == -INFINITY) ? 0.0f : expf(ms - M);
            num = fmaf(__ldcg(pb + (size_t)s2 * (hd + 2) + d), w, num);
            den = fmaf(__ldcg(pb + (size_t)s2 * (hd + 2) + hd + 1), w, den);
        }
        p.out[(size_t)h * hd + d] = den > 0.0f ? num / den : 0.0f;
    }
    if (tid == 0)
        p.counters[kvh] = 0u;
}

} // namespace aaedn_dev
