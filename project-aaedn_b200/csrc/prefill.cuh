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

#include <climits>

#include "common.cuh"
#include "gemm_tc.h"  // tc_kpos
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

// One CTA per row m < M_pad: parts[q][m][tc_kpos(k)] (q = 0, 1, 2: the bf16
// parts of x * rms * g, src/rmsnorm.cpp:34-43); rows m >= M are zero.
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
        const int kp = tc_kpos(k); // the GEMM operand's K order
        p0[kp] = h;
        p0[kp + plane] = md;
        p0[kp + 2 * plane] = __float2bfloat16_rn(r1 - __bfloat162float(md));
    }
}

constexpr int PF_ATTN_WARPS = 4;

// Causal attention of rows t < n for query head blockIdx.x: one warp per
// row. Row t is the token at position pos0 + t of the sequence whose pages
// page_table lists (a prefill chunk; batched decode rows use
// attn_decode_kernel). Keys are taken 32 at a time,
// lane j scoring key s0 + j against q (held in shared memory); the batch's
// softmax weights then scale the V rows with lanes over the head dims; the
// softmax is carried online across batches (running max and sum). fp32,
// expf (D4). out[t][h * hd + d]; head_dim a multiple of 32, <= 256.
__global__ void __launch_bounds__(PF_ATTN_WARPS * 32) attn_prefill_kernel(
    const float* __restrict__ q, size_t ldq, const float* __restrict__ k_layer, const float* __restrict__ v_layer,
    const int* __restrict__ page_table_base, int page_size, int n_heads, int n_kv, int hd, int pos0, int n,
    float scale, float* __restrict__ out, size_t ldo)
{
    __shared__ __align__(16) float qs[PF_ATTN_WARPS][256];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int h = blockIdx.x, t = blockIdx.y * PF_ATTN_WARPS + warp;
    if (t >= n)
        return;
    const int kvh = h / (n_heads / n_kv);
    const int pos = pos0 + t, nkeys = pos + 1;
    const int* page_table = page_table_base;
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
        // the batch's V rows 8 at a time, every load of a group issued
        // before its first use; keys in ascending order into each sum
        const int nb = min(32, nkeys - s0);
        for (int j0 = 0; j0 < nb; j0 += 8)
        {
            float wj[8], vv[8][8];
#pragma unroll
            for (int u = 0; u < 8; ++u)
            {
                const int j = j0 + u;
                wj[u] = __shfl_sync(0xffffffffu, w, j & 31);
                const float* vr = nullptr;
                if (j < nb)
                {
                    const int sj = s0 + j;
                    const int page = page_table[sj / page_size];
                    vr = v_layer + (((size_t)page * n_kv + kvh) * page_size + (sj % page_size)) * hd;
                }
#pragma unroll
                for (int i = 0; i < 8; ++i)
                    vv[u][i] = (vr && i < dpl) ? vr[lane + 32 * i] : 0.0f;
            }
#pragma unroll
            for (int u = 0; u < 8; ++u)
                if (j0 + u < nb)
#pragma unroll
                    for (int i = 0; i < 8; ++i)
                        if (i < dpl)
                            acc[i] = fmaf(wj[u], vv[u][i], acc[i]);
        }
    }
    const float inv = 1.0f / lrun;
    float* o = out + (size_t)t * ldo + (size_t)h * hd;
#pragma unroll
    for (int i = 0; i < 8; ++i)
        if (i < dpl)
            o[lane + 32 * i] = acc[i] * inv;
}

// ---------------------------------------------------------------------------
// Causal attention of a prefill chunk, tiled: CTA (query head h, 64 query
// rows), 8 warps of 8 rows each; the keys come in tiles of 32 (K and V rows
// of one page, copied with cp.async into padded shared memory, the next tile
// in flight while this one is used), so each K/V row is read once per 64
// query rows instead of once per row. A warp scores its 8 rows against the
// tile with lanes over keys (q rows broadcast from shared memory), carries
// the online softmax per row (running max warp-wide, each lane its share of
// the running sum), then accumulates P V with lanes over head dims (4 each).
// fp32, expf (D4); head_dim a multiple of 4, <= 128; page_size a multiple
// of 32. out[t][h * hd + d].
// ---------------------------------------------------------------------------
constexpr int PFT_Q = 64, PFT_K = 32, PFT_WARPS = 8, PFT_RW = PFT_Q / PFT_WARPS, PFT_LD = 128 + 4;

inline size_t attn_prefill_tiled_smem_bytes() { return ((size_t)PFT_Q * PFT_LD + 4 * PFT_K * PFT_LD + PFT_WARPS * PFT_RW * PFT_K) * 4; }

__global__ void __launch_bounds__(PFT_WARPS * 32, 2) attn_prefill_tiled_kernel(
    const float* __restrict__ q, size_t ldq, const float* __restrict__ k_layer, const float* __restrict__ v_layer,
    const int* __restrict__ page_table, int page_size, int n_heads, int n_kv, int hd, int pos0, int n, float scale,
    float* __restrict__ out, size_t ldo)
{
    extern __shared__ __align__(16) float pft[];
    float* Qs = pft;                                  // [64][LD]
    float* KV = Qs + PFT_Q * PFT_LD;                  // [2 buffers][K, V][32][LD]
    float* Ps = KV + 4 * PFT_K * PFT_LD;              // [8 warps][8 rows][32]
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int h = blockIdx.x, kvh = h / (n_heads / n_kv), r0 = blockIdx.y * PFT_Q;
    const int hd4 = hd >> 2;
    // the chunk's rows r0..: q into shared memory (rows past n are zero)
    for (int i = tid; i < PFT_Q * hd4; i += PFT_WARPS * 32)
    {
        const int r = i / hd4, c = i - r * hd4;
        const float4 v = r0 + r < n ? *reinterpret_cast<const float4*>(q + (size_t)(r0 + r) * ldq + (size_t)h * hd + 4 * c)
                                    : make_float4(0.f, 0.f, 0.f, 0.f);
        *reinterpret_cast<float4*>(Qs + r * PFT_LD + 4 * c) = v;
    }
    const int last_pos = pos0 + min(n, r0 + PFT_Q) - 1; // keys 0..last_pos
    const int ntiles = last_pos / PFT_K + 1;
    auto issue = [&](int tile, int buf) {
        const int k0 = tile * PFT_K;
        const int page = page_table[k0 / page_size];
        const size_t base = (((size_t)page * n_kv + kvh) * page_size + (k0 % page_size)) * hd;
        float* Kb = KV + (size_t)buf * 2 * PFT_K * PFT_LD;
        float* Vb = Kb + PFT_K * PFT_LD;
        for (int i = tid; i < PFT_K * hd4; i += PFT_WARPS * 32)
        {
            const int r = i / hd4, c = i - r * hd4;
            const uint32_t ok = k0 + r <= last_pos ? 16u : 0u; // rows past the last key: zero
            cp_async_16(Kb + r * PFT_LD + 4 * c, k_layer + base + (size_t)r * hd + 4 * c, ok);
            cp_async_16(Vb + r * PFT_LD + 4 * c, v_layer + base + (size_t)r * hd + 4 * c, ok);
        }
        cp_async_commit();
    };
    issue(0, 0);
    float m[PFT_RW], l[PFT_RW];
    float4 acc[PFT_RW];
#pragma unroll
    for (int i = 0; i < PFT_RW; ++i)
    {
        m[i] = -INFINITY;
        l[i] = 0.0f;
        acc[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    const int wrow0 = r0 + warp * PFT_RW; // this warp's first row
    float* Pw = Ps + warp * PFT_RW * PFT_K;
    for (int t = 0; t < ntiles; ++t)
    {
        if (t + 1 < ntiles)
        {
            issue(t + 1, (t + 1) & 1);
            cp_async_wait<1>();
        }
        else
            cp_async_wait<0>();
        __syncthreads();
        const float* Kb = KV + (size_t)(t & 1) * 2 * PFT_K * PFT_LD;
        const float* Vb = Kb + PFT_K * PFT_LD;
        const int kpos = t * PFT_K + lane;
        // rows of this warp that see any key of the tile (warp-uniform)
        if (pos0 + wrow0 + PFT_RW - 1 >= t * PFT_K && wrow0 < n)
        {
            float sc[PFT_RW];
#pragma unroll
            for (int i = 0; i < PFT_RW; ++i)
                sc[i] = 0.0f;
            const float* kr = Kb + lane * PFT_LD;
            const float* qw = Qs + (warp * PFT_RW) * PFT_LD;
            for (int c = 0; c < hd4; ++c)
            {
                const float4 kf = *reinterpret_cast<const float4*>(kr + 4 * c);
#pragma unroll
                for (int i = 0; i < PFT_RW; ++i)
                {
                    const float4 qf = *reinterpret_cast<const float4*>(qw + i * PFT_LD + 4 * c);
                    sc[i] = fmaf(qf.x, kf.x, sc[i]);
                    sc[i] = fmaf(qf.y, kf.y, sc[i]);
                    sc[i] = fmaf(qf.z, kf.z, sc[i]);
                    sc[i] = fmaf(qf.w, kf.w, sc[i]);
                }
            }
#pragma unroll
            for (int i = 0; i < PFT_RW; ++i)
            {
                const int rpos = pos0 + wrow0 + i;
                const bool live = wrow0 + i < n && kpos <= rpos;
                const float s = live ? sc[i] * scale : -INFINITY; // src/attention.cpp:36-41
                const float bm = warp_max(s);
                const float mn = fmaxf(m[i], bm);
                float p = 0.0f, corr = 1.0f;
                if (mn != -INFINITY)
                {
                    corr = (m[i] == -INFINITY) ? 0.0f : expf(m[i] - mn);
                    p = live ? expf(s - mn) : 0.0f;
                    m[i] = mn;
                }
                l[i] = l[i] * corr + p;
                acc[i].x *= corr;
                acc[i].y *= corr;
                acc[i].z *= corr;
                acc[i].w *= corr;
                Pw[i * PFT_K + lane] = p;
            }
            __syncwarp();
            if (lane < hd4)
                for (int j = 0; j < PFT_K; ++j)
                {
                    const float4 vf = *reinterpret_cast<const float4*>(Vb + j * PFT_LD + 4 * lane);
#pragma unroll
                    for (int i = 0; i < PFT_RW; ++i)
                    {
                        const float pj = Pw[i * PFT_K + j];
                        acc[i].x = fmaf(pj, vf.x, acc[i].x);
                        acc[i].y = fmaf(pj, vf.y, acc[i].y);
                        acc[i].z = fmaf(pj, vf.z, acc[i].z);
                        acc[i].w = fmaf(pj, vf.w, acc[i].w);
                    }
                }
            __syncwarp();
        }
        __syncthreads(); // the buffer is refilled two tiles on
    }
#pragma unroll
    for (int i = 0; i < PFT_RW; ++i)
    {
        const float lt = warp_sum(l[i]);
        if (wrow0 + i < n && lane < hd4)
        {
            const float inv = 1.0f / lt;
            *reinterpret_cast<float4*>(out + (size_t)(wrow0 + i) * ldo + (size_t)h * hd + 4 * lane) =
                make_float4(acc[i].x * inv, acc[i].y * inv, acc[i].z * inv, acc[i].w * inv);
        }
    }
}

// ---------------------------------------------------------------------------
// lm_head over several rows (batched decode): the final RMSNorm of each row
// (src/transformer.cpp:230), the fp32 product with the [vocab][dim] lm_head
// (:232-238) and each row's greedy token (argmax, ties to the lowest id).
// ---------------------------------------------------------------------------

// out[m][k] = x[m][k] * rms(x[m]) * g[k]; one CTA per row.
__global__ void __launch_bounds__(256) pf_rmsnorm_rows_kernel(const float* __restrict__ x, int D,
                                                              const float* __restrict__ gain, float eps,
                                                              float* __restrict__ out)
{
    __shared__ float scratch[64];
    const float* xr = x + (size_t)blockIdx.x * D;
    float ss = 0.0f;
    for (int k = threadIdx.x; k < D; k += blockDim.x)
        ss = fmaf(xr[k], xr[k], ss);
    ss = block_sum(ss, scratch);
    const float rms = 1.0f / sqrtf(__fadd_rn(__fdiv_rn(ss, (float)D), eps));
    for (int k = threadIdx.x; k < D; k += blockDim.x)
        out[(size_t)blockIdx.x * D + k] = __fmul_rn(__fmul_rn(xr[k], rms), gain[k]);
}

// Greedy-token partials: a CTA's best (value, id) per activation row over its
// vocabulary rows, ties to the lowest id; argmax_parts_kernel takes the best
// of a row's partials in order.
__device__ __forceinline__ void lr_better(float& v, int& i, float ov, int oi)
{
    if (ov > v || (ov == v && oi < i))
    {
        v = ov;
        i = oi;
    }
}

constexpr int LR_BM = 32, LR_BN = 128, LR_BK = 32, LR_LD = LR_BK + 4, LR_STAGES = 4;

inline size_t lm_rows_smem_bytes() { return (size_t)LR_STAGES * (LR_BN + LR_BM) * LR_LD * 4; }

// out[m * ldo + v] = sum_k x[m][k] * w[v][k] for m < M (<= 32 a launch row
// tile, blockIdx.y), v < V, and the CTA's greedy partial per row into
// part_val / part_idx [M][gridDim.x]. A CTA of 256 threads owns 128
// vocabulary rows x 32 activation rows (4 x 4 per thread), K in slices of
// 32 through a 4-stage cp.async ring (rows of 16-byte pieces, padded), k
// ascending in every sum. D a multiple of 32.
__global__ void __launch_bounds__(256, 2) lm_rows_kernel(const float* __restrict__ x, int M, int D,
                                                         const float* __restrict__ w, int V, float* __restrict__ out,
                                                         size_t ldo, float* __restrict__ part_val,
                                                         int* __restrict__ part_idx)
{
    extern __shared__ __align__(16) float lr[];
    const int tid = threadIdx.x, tm = tid & 7, tn = tid >> 3;
    const int v0 = blockIdx.x * LR_BN, m0 = blockIdx.y * LR_BM;
    auto ws = [&](int s) { return lr + (size_t)s * (LR_BN + LR_BM) * LR_LD; };
    auto xs = [&](int s) { return ws(s) + LR_BN * LR_LD; };
    const int nk = D / LR_BK;
    auto issue = [&](int kb, int s) {
        // 128 w rows and 32 x rows of 32 floats: 8 pieces of 16 bytes each
        for (int i = tid; i < (LR_BN + LR_BM) * 8; i += 256)
        {
            const int r = i >> 3, c = i & 7;
            if (r < LR_BN)
            {
                const int v = v0 + r;
                const float* src = w + (size_t)min(v, V - 1) * D + kb * LR_BK + 4 * c;
                cp_async_16(ws(s) + r * LR_LD + 4 * c, src, v < V ? 16u : 0u);
            }
            else
            {
                const int m = m0 + r - LR_BN;
                const float* src = x + (size_t)min(m, M - 1) * D + kb * LR_BK + 4 * c;
                cp_async_16(xs(s) + (r - LR_BN) * LR_LD + 4 * c, src, m < M ? 16u : 0u);
            }
        }
        cp_async_commit();
    };
#pragma unroll
    for (int s = 0; s < LR_STAGES - 1; ++s)
    {
        if (s < nk)
            issue(s, s);
        else
            cp_async_commit();
    }
    float acc[4][4] = {}; // [vocab i][row j]
    for (int kb = 0; kb < nk; ++kb)
    {
        cp_async_wait<LR_STAGES - 2>();
        __syncthreads();
        if (kb + LR_STAGES - 1 < nk)
            issue(kb + LR_STAGES - 1, (kb + LR_STAGES - 1) % LR_STAGES);
        else
            cp_async_commit();
        const float* W = ws(kb % LR_STAGES);
        const float* X = xs(kb % LR_STAGES);
#pragma unroll
        for (int k = 0; k < LR_BK; k += 4)
        {
            float4 a[4], b[4];
#pragma unroll
            for (int i = 0; i < 4; ++i)
                a[i] = *reinterpret_cast<const float4*>(W + (tn * 4 + i) * LR_LD + k);
#pragma unroll
            for (int j = 0; j < 4; ++j)
                b[j] = *reinterpret_cast<const float4*>(X + (tm * 4 + j) * LR_LD + k);
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j)
                {
                    acc[i][j] = fmaf(a[i].x, b[j].x, acc[i][j]);
                    acc[i][j] = fmaf(a[i].y, b[j].y, acc[i][j]);
                    acc[i][j] = fmaf(a[i].z, b[j].z, acc[i][j]);
                    acc[i][j] = fmaf(a[i].w, b[j].w, acc[i][j]);
                }
        }
    }
    cp_async_wait<0>();
    __syncthreads();
    // logits, and each row's best over this CTA's 128 vocabulary rows
    float* sbv = lr;                                  // [32 tn][32 rows]
    int* sbi = reinterpret_cast<int*>(lr + 32 * LR_BM);
#pragma unroll
    for (int j = 0; j < 4; ++j)
    {
        const int m = m0 + tm * 4 + j;
        float bv = -INFINITY;
        int bi = INT_MAX;
#pragma unroll
        for (int i = 0; i < 4; ++i)
        {
            const int v = v0 + tn * 4 + i;
            if (v < V && m < M)
            {
                out[(size_t)m * ldo + v] = acc[i][j];
                lr_better(bv, bi, acc[i][j], v);
            }
        }
        sbv[tn * LR_BM + tm * 4 + j] = bv;
        sbi[tn * LR_BM + tm * 4 + j] = bi;
    }
    __syncthreads();
    if (tid < LR_BM && m0 + tid < M)
    {
        float bv = -INFINITY;
        int bi = INT_MAX;
        for (int t = 0; t < 32; ++t)
            lr_better(bv, bi, sbv[t * LR_BM + tid], sbi[t * LR_BM + tid]);
        part_val[(size_t)(m0 + tid) * gridDim.x + blockIdx.x] = bv;
        part_idx[(size_t)(m0 + tid) * gridDim.x + blockIdx.x] = bi;
    }
}

constexpr int LF_MAXM = 4, LF_WARPS = 8;

// The same product for at most 4 activation rows (a prefill's last row):
// every warp streams whole vocabulary rows (lanes over D, 16-byte loads)
// against the rows held in shared memory; per-CTA greedy partials as above.
// D a multiple of 128.
__global__ void __launch_bounds__(LF_WARPS * 32) lm_rows_few_kernel(const float* __restrict__ x, int M, int D,
                                                                    const float* __restrict__ w, int V,
                                                                    float* __restrict__ out, size_t ldo,
                                                                    float* __restrict__ part_val,
                                                                    int* __restrict__ part_idx)
{
    extern __shared__ __align__(16) float xsm[]; // [M][D]
    __shared__ float sbv[LF_WARPS][LF_MAXM];
    __shared__ int sbi[LF_WARPS][LF_MAXM];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    for (int i = tid; i < M * D / 4; i += blockDim.x)
        reinterpret_cast<float4*>(xsm)[i] = reinterpret_cast<const float4*>(x)[i];
    __syncthreads();
    float bv[LF_MAXM], tmp[LF_MAXM];
    int bi[LF_MAXM];
#pragma unroll
    for (int j = 0; j < LF_MAXM; ++j)
    {
        bv[j] = -INFINITY;
        bi[j] = INT_MAX;
    }
    const int per = (V + gridDim.x - 1) / gridDim.x, v_begin = blockIdx.x * per, v_end = min(V, v_begin + per);
    for (int v = v_begin + warp; v < v_end; v += LF_WARPS)
    {
        const float4* wr = reinterpret_cast<const float4*>(w + (size_t)v * D);
#pragma unroll
        for (int j = 0; j < LF_MAXM; ++j)
            tmp[j] = 0.0f;
        for (int c = lane; c < D / 4; c += 32)
        {
            const float4 a = __ldcs(wr + c);
#pragma unroll
            for (int j = 0; j < LF_MAXM; ++j)
                if (j < M)
                {
                    const float4 b = reinterpret_cast<const float4*>(xsm + (size_t)j * D)[c];
                    tmp[j] = fmaf(a.x, b.x, tmp[j]);
                    tmp[j] = fmaf(a.y, b.y, tmp[j]);
                    tmp[j] = fmaf(a.z, b.z, tmp[j]);
                    tmp[j] = fmaf(a.w, b.w, tmp[j]);
                }
        }
#pragma unroll
        for (int j = 0; j < LF_MAXM; ++j)
            if (j < M)
            {
                const float s = warp_sum(tmp[j]);
                if (lane == 0)
                {
                    out[(size_t)j * ldo + v] = s;
                    lr_better(bv[j], bi[j], s, v);
                }
            }
    }
    if (lane == 0)
#pragma unroll
        for (int j = 0; j < LF_MAXM; ++j)
        {
            sbv[warp][j] = bv[j];
            sbi[warp][j] = bi[j];
        }
    __syncthreads();
    if (tid < M)
    {
        float b = -INFINITY;
        int i = INT_MAX;
        for (int w8 = 0; w8 < LF_WARPS; ++w8)
            lr_better(b, i, sbv[w8][tid], sbi[w8][tid]);
        part_val[(size_t)tid * gridDim.x + blockIdx.x] = b;
        part_idx[(size_t)tid * gridDim.x + blockIdx.x] = i;
    }
}

// next[m] = the best of row m's n_parts partials (ties to the lowest id);
// one warp per row.
__global__ void __launch_bounds__(256) argmax_parts_kernel(const float* __restrict__ part_val,
                                                           const int* __restrict__ part_idx, int n_parts, int M,
                                                           uint32_t* __restrict__ next)
{
    const int m = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (m >= M)
        return;
    float bv = -INFINITY;
    int bi = INT_MAX;
    for (int c = lane; c < n_parts; c += 32)
        lr_better(bv, bi, part_val[(size_t)m * n_parts + c], part_idx[(size_t)m * n_parts + c]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
        lr_better(bv, bi, __shfl_xor_sync(0xffffffffu, bv, o), __shfl_xor_sync(0xffffffffu, bi, o));
    if (lane == 0)
        next[m] = bi == INT_MAX ? 0u : (uint32_t)bi;
}

} // namespace aaedn_dev
