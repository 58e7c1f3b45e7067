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
//
// Memory-level parallelism (the K/V stream is HBM-bound): a CTA stages its
// rows 64 tokens at a time in shared memory with asynchronous 16-byte copies
// (every row of K and V of the chunk in flight at once). Rows written in
// earlier decode steps are requested before waiting for the previous kernel,
// so their latency overlaps it; across chunks the softmax is carried online
// (running max and sum, rescaled per chunk).
#pragma once

#include "gemv_q4.cuh"

namespace aaedn_dev
{

constexpr int ATTN_THREADS = 256;
constexpr int ATTN_WARPS = ATTN_THREADS / 32;
constexpr int ATTN_MAX_SEG = 64;
constexpr int ATTN_MAX_HD = 256;
constexpr int ATTN_MAX_G = 8; // query heads per kv head (template values 1, 2, 4, 8)

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

// Score rows are padded to a multiple of 4 floats so the float4 regions
// after them stay 16-byte aligned.
__host__ __device__ inline int attn_score_stride(int max_tok) { return (max_tok + 3) & ~3; }

constexpr int ATTN_CHUNK = 64; // tokens staged in shared memory at a time

// Rows of K and V in shared memory are padded by 16 bytes so that threads
// reading different rows at the same offset hit different banks.
__host__ __device__ inline int attn_row_stride(int hd) { return hd + 4; }

inline size_t attn_smem_bytes(int G, int hd, int /*max_tok*/)
{
    // K and V chunks [CH][hd+4], q [G][hd], scores [G][CH], per-slice V sums
    // [8][G][hd], per-head running max/sum/rescale [3][G]
    return ((size_t)2 * ATTN_CHUNK * attn_row_stride(hd) + (size_t)G * hd + (size_t)G * ATTN_CHUNK +
            (size_t)8 * G * hd + 3 * ATTN_MAX_G + 8) *
           4;
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

// G: query heads per kv head; HDM: bound on head_dim (128 or 256).
template <int MODE, int G, int HDM>
__global__ void __launch_bounds__(ATTN_THREADS) attn_split_kernel(const AttnParams p)
{
    extern __shared__ __align__(16) float asmem[];
    pdl_launch_dependents();
    const int kvh = blockIdx.x, split = blockIdx.y, S = p.S;
    const int hd = p.head_dim, hd4 = hd >> 2, rs = attn_row_stride(hd);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    // The position only changes at the end of a decode step (lm_head), so it
    // can be read before waiting for the previous kernel.
    int L = (MODE == 1) ? (int)p.state->pos + 1 : p.len_static;
    if (L > p.max_len)
        L = p.max_len;
    const int t0 = (int)(((long long)L * split) / S);
    const int t1 = (int)(((long long)L * (split + 1)) / S);
    // The row of the current position is written by the previous kernel;
    // every other row was written in earlier steps.
    const int cur = (MODE == 1) ? L - 1 : -1;

    float* ks = asmem;                           // [CH][rs]
    float* vs = ks + ATTN_CHUNK * rs;            // [CH][rs]
    float* qs = vs + ATTN_CHUNK * rs;            // [G][hd]
    float* sc = qs + G * hd;                     // [G][CH]
    float* vred = sc + G * ATTN_CHUNK;           // [8][G][hd]
    float* run = vred + 8 * G * hd;              // [3][G]: running max, sum, rescale

    auto stage = [&](int c0, int c1) { // async copies of rows [c0, c1) except cur
        const int n = c1 - c0;
        for (int i = tid; i < n * hd4; i += ATTN_THREADS)
        {
            const int j = i / hd4, c = i - j * hd4, tk = c0 + j;
            if (tk == cur)
                continue;
            const size_t ro = attn_row<MODE>(p, tk, kvh);
            cp_async_16(ks + j * rs + 4 * c, p.k + ro + 4 * c, 16u);
            cp_async_16(vs + j * rs + 4 * c, p.v + ro + 4 * c, 16u);
        }
        cp_async_commit();
    };

    const int c_end0 = t0 + ATTN_CHUNK < t1 ? t0 + ATTN_CHUNK : t1;
    if (t1 > t0)
        stage(t0, c_end0);
    pdl_wait();
    for (int i = tid; i < G * hd; i += ATTN_THREADS)
        qs[i] = p.q[(size_t)kvh * G * hd + i];
    if (tid < G)
    {
        run[tid] = -INFINITY;
        run[G + tid] = 0.0f;
    }

    // per-thread V accumulators: chunk c4 = tid % 32 of the row (float4),
    // token slice z = tid / 32
    constexpr int NC = HDM / 128;
    float4 acc[G][NC];
#pragma unroll
    for (int gi = 0; gi < G; ++gi)
#pragma unroll
        for (int c = 0; c < NC; ++c)
            acc[gi][c] = make_float4(0.f, 0.f, 0.f, 0.f);

    for (int c0 = t0; c0 < t1; c0 += ATTN_CHUNK)
    {
        const int c1 = c0 + ATTN_CHUNK < t1 ? c0 + ATTN_CHUNK : t1;
        const int n = c1 - c0;
        if (c0 != t0)
            stage(c0, c1);
        if (cur >= c0 && cur < c1) // the fresh row, after the previous kernel
            for (int c = tid; c < hd4; c += ATTN_THREADS)
            {
                const size_t ro = attn_row<MODE>(p, cur, kvh);
                reinterpret_cast<float4*>(ks + (cur - c0) * rs)[c] = reinterpret_cast<const float4*>(p.k + ro)[c];
                reinterpret_cast<float4*>(vs + (cur - c0) * rs)[c] = reinterpret_cast<const float4*>(p.v + ro)[c];
            }
        cp_async_wait<0>();
        __syncthreads();

        // scores: one thread per (token, query head)
        for (int idx = tid; idx < n * G; idx += ATTN_THREADS)
        {
            const int j = idx / G, gi = idx - j * G;
            const float4* kr = reinterpret_cast<const float4*>(ks + j * rs);
            const float4* qr = reinterpret_cast<const float4*>(qs + gi * hd);
            float dot = 0.0f;
            for (int c = 0; c < hd4; ++c)
            {
                const float4 a = qr[c], b = kr[c];
                dot = fmaf(a.x, b.x, dot);
                dot = fmaf(a.y, b.y, dot);
                dot = fmaf(a.z, b.z, dot);
                dot = fmaf(a.w, b.w, dot);
            }
            sc[gi * ATTN_CHUNK + j] = dot * p.scale; // src/attention.cpp:42
        }
        __syncthreads();

        // running max / exp / sum per query head (src/attention.cpp:46-59)
        for (int gi = warp; gi < G; gi += ATTN_WARPS)
        {
            float mx = -INFINITY;
            for (int j = lane; j < n; j += 32)
                mx = fmaxf(mx, sc[gi * ATTN_CHUNK + j]);
            mx = warp_max(mx);
            const float m_old = run[gi];
            const float m_new = fmaxf(m_old, mx);
            float sum = 0.0f;
            for (int j = lane; j < n; j += 32)
            {
                const float e = expf(sc[gi * ATTN_CHUNK + j] - m_new);
                sc[gi * ATTN_CHUNK + j] = e;
                sum += e;
            }
            sum = warp_sum(sum);
            if (lane == 0)
            {
                const float resc = (m_old == -INFINITY) ? 0.0f : expf(m_old - m_new);
                run[gi] = m_new;
                run[G + gi] = run[G + gi] * resc + sum;
                run[2 * G + gi] = resc;
            }
        }
        __syncthreads();

        // V: thread (slice z, chunk c4) sums tokens z, z+8, ... of the chunk
        {
            const int z = tid >> 5, c4 = tid & 31;
#pragma unroll
            for (int gi = 0; gi < G; ++gi)
            {
                const float rsc = run[2 * G + gi];
#pragma unroll
                for (int c = 0; c < NC; ++c)
                {
                    acc[gi][c].x *= rsc;
                    acc[gi][c].y *= rsc;
                    acc[gi][c].z *= rsc;
                    acc[gi][c].w *= rsc;
                }
            }
            for (int j = z; j < n; j += 8)
            {
#pragma unroll
                for (int c = 0; c < NC; ++c)
                {
                    const int ch = c4 + 32 * c;
                    if (ch < hd4)
                    {
                        const float4 vv = reinterpret_cast<const float4*>(vs + j * rs)[ch];
#pragma unroll
                        for (int gi = 0; gi < G; ++gi)
                        {
                            const float e = sc[gi * ATTN_CHUNK + j];
                            acc[gi][c].x = fmaf(e, vv.x, acc[gi][c].x);
                            acc[gi][c].y = fmaf(e, vv.y, acc[gi][c].y);
                            acc[gi][c].z = fmaf(e, vv.z, acc[gi][c].z);
                            acc[gi][c].w = fmaf(e, vv.w, acc[gi][c].w);
                        }
                    }
                }
            }
        }
        __syncthreads(); // the chunk buffers are rewritten next
    }
    {
        const int z = tid >> 5, c4 = tid & 31;
#pragma unroll
        for (int gi = 0; gi < G; ++gi)
#pragma unroll
            for (int c = 0; c < NC; ++c)
            {
                const int ch = c4 + 32 * c;
                if (ch < hd4)
                    reinterpret_cast<float4*>(vred + ((size_t)z * G + gi) * hd)[ch] = acc[gi][c];
            }
    }
    __syncthreads();
    for (int i = tid; i < G * hd; i += ATTN_THREADS)
    {
        const int gi = i / hd, d = i - gi * hd;
        float o = 0.0f;
        for (int z = 0; z < 8; ++z) // fixed order
            o += vred[((size_t)z * G + gi) * hd + d];
        const int h = kvh * G + gi;
        float* pp = p.part + ((size_t)h * S + split) * (hd + 2);
        pp[d] = o;
        if (d == 0)
        {
            pp[hd] = (t1 > t0) ? run[gi] : -INFINITY;
            pp[hd + 1] = run[G + gi];
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

namespace aaedn_dev
{

template <int MODE, int G, int HDM>
inline cudaError_t attn_launch_one(const AttnParams& p, dim3 grid, size_t smem, cudaStream_t st, bool pdl)
{
    return launch_kernel(attn_split_kernel<MODE, G, HDM>, grid, dim3(ATTN_THREADS), smem, st, pdl, p);
}

// Launches the instantiation for G = n_heads / n_kv (1, 2, 4 or 8).
template <int MODE>
inline int attn_launch(const AttnParams& p, dim3 grid, size_t smem, cudaStream_t st, bool pdl = false)
{
    const int G = p.n_heads / p.n_kv;
    const bool big = p.head_dim > 128;
    cudaError_t e;
    switch (G)
    {
    case 1: e = big ? attn_launch_one<MODE, 1, 256>(p, grid, smem, st, pdl) : attn_launch_one<MODE, 1, 128>(p, grid, smem, st, pdl); break;
    case 2: e = big ? attn_launch_one<MODE, 2, 256>(p, grid, smem, st, pdl) : attn_launch_one<MODE, 2, 128>(p, grid, smem, st, pdl); break;
    case 4: e = big ? attn_launch_one<MODE, 4, 256>(p, grid, smem, st, pdl) : attn_launch_one<MODE, 4, 128>(p, grid, smem, st, pdl); break;
    case 8: e = big ? attn_launch_one<MODE, 8, 256>(p, grid, smem, st, pdl) : attn_launch_one<MODE, 8, 128>(p, grid, smem, st, pdl); break;
    default: return set_error(AAEDN_EUNSUPPORTED, "attention: %d query heads per kv head (1, 2, 4 or 8)", G);
    }
    if (e != cudaSuccess)
        return set_error(AAEDN_ECUDA, "launch of attn_split_kernel failed: %s", cudaGetErrorString(e));
    count_launch();
    return AAEDN_OK;
}

template <int MODE, int G>
inline int attn_set_attrs_g()
{
    AAEDN_CUDA_TRY(cudaFuncSetAttribute(attn_split_kernel<MODE, G, 128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        200 * 1024));
    AAEDN_CUDA_TRY(cudaFuncSetAttribute(attn_split_kernel<MODE, G, 256>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        200 * 1024));
    return AAEDN_OK;
}

template <int MODE>
inline int attn_set_attrs()
{
    int rc = attn_set_attrs_g<MODE, 1>();
    if (!rc)
        rc = attn_set_attrs_g<MODE, 2>();
    if (!rc)
        rc = attn_set_attrs_g<MODE, 4>();
    if (!rc)
        rc = attn_set_attrs_g<MODE, 8>();
    return rc;
}

} // namespace aaedn_dev
