// gemv_q4.cuh — block-quantized (4-bit codes, one scale per 32 codes of a
// row) matrix-vector product for M <= 8 activation rows, fp32 in and out.
//
// Replaces the scalar dequant + GEMV loops of src/transformer.cpp:155-215,
// src/ffn.cpp:36-75 and the intended product of src/fused_matmul.cpp:70-169.
//
// Design (HBM-bound: 0.5625 B per weight, ~12 T weights/s at the measured
// HBM peak, i.e. ~3 issue slots per weight at most):
//  * the weights are streamed once from HBM in the reference layout ([N][K]
//    rows, 16 bytes of codes per 32-code block, flat-order scales) with
//    16-byte non-temporal loads; each lane of a quad reads one whole block of
//    its two rows (g, g+8), so every load is a full aligned 16-byte vector;
//  * codes are turned into bf16 values 16 + c with one shift and one LOP3 per
//    two codes (exact: 4-bit integers are exact in bf16);
//  * the tensor core (mma.sync m16n8k16 bf16 -> fp32) is used as the dot
//    product engine: A = 16 weight rows x 16 codes, B columns = 4 quant
//    blocks x 2 parts of the activation (x = hi + lo, both bf16, so x is
//    carried to 2^-18 relative), so each lane's fp32 accumulators hold the
//    per-(row, block) partial sums its own block needs;
//  * the per-block epilogue removes the +16 bias with a precomputed
//    16*sum(x) per block and applies the block scale in fp32;
//  * RMSNorm (prologue), RoPE + KV-cache append, SwiGLU and the residual add
//    (epilogues) are fused for the decode path.
#pragma once

#include "common.cuh"

namespace aaedn_dev
{

enum
{
    PRO_PLAIN = 0,
    PRO_RMSNORM = 1,
    PRO_EMBED_RMSNORM = 2,
};

enum
{
    EPI_STORE = 0,
    EPI_ACCUM = 1,
    EPI_RESIDUAL = 2,
    EPI_QKV_ROPE = 3,
    EPI_SWIGLU = 4,
};

// Decode state that lives on the device so a whole step can be replayed as
// one CUDA graph: the position, where the next input token comes from and
// the greedy output.
struct DecodeState
{
    uint32_t pos;        // position of the token processed by this step
    uint32_t n_prompt;   // prompt[0..n_prompt) are forced inputs
    uint32_t next_token; // argmax of the previous step
    uint32_t lm_counter; // last-CTA counter of the lm_head kernel (self-resetting)
    uint32_t err;        // sticky device-side error flag
    uint32_t pad[3];
};

struct GemvParams
{
    const uint8_t* w;  // codes, row n at byte n*ldb/2
    const uint16_t* s; // scales, row n at n*ldb/32
    size_t ldb;        // codes per weight row (multiple of 32)
    int N;             // output rows
    int K;             // valid codes per row (multiple of 32)
    int kt0, kt1;      // 128-code tiles of K handled by this launch
    const float* x;    // activations [NM][lda]
    size_t lda;
    float* y; // output [NM][ldc]
    size_t ldc;
    // RMSNorm prologue
    const float* gain;
    float eps;
    // embedding prologue (decode step input)
    const float* embedding;
    const uint32_t* prompt;
    DecodeState* state;
    float* hidden_out;
    // QKV epilogue: RoPE on q/k rows, k/v appended to the paged cache
    int q_rows, kv_rows, head_dim, n_kv, page_size;
    int max_pos; // cache capacity: positions >= max_pos are not written
    float* qbuf;
    float* k_layer;
    float* v_layer;
    const int* page_table;
    const float* rope_cos;
    const float* rope_sin;
    // SwiGLU epilogue
    float* act;
};

constexpr int GEMV_WARPS = 8;

// Dynamic shared memory of one CTA.
inline size_t gemv_smem_bytes(int nm, int ntile, int R, int S)
{
    return (size_t)nm * ntile * 512 + (size_t)nm * ntile * 16 + (size_t)nm * S * R * 16 * 4 + 64 * 4;
}

__device__ __forceinline__ uint32_t u4get(const uint4& v, int q)
{
    return q == 0 ? v.x : (q == 1 ? v.y : (q == 2 ? v.z : v.w));
}

// Block-wide sum; every thread receives the result. scratch >= 33 floats.
__device__ __forceinline__ float block_sum(float v, float* scratch)
{
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    v = warp_sum(v);
    __syncthreads();
    if (lane == 0)
        scratch[warp] = v;
    __syncthreads();
    float t = 0.0f;
    for (int i = 0; i < nw; ++i) // fixed order: deterministic
        t += scratch[i];
    return t;
}

// Builds the B-operand fragments of the activations for tiles [kt0, kt1):
// frag[((m*ntile + tt)*4 + q)*8 + la] holds, for lane slot la = 2*tp + p
// (block tp of the tile, part p), the 4 bf16x2 registers of mmas 2q and
// 2q+1: (x[8q+0],x[8q+4]), (x[8q+1],x[8q+5]), (x[8q+2],x[8q+6]),
// (x[8q+3],x[8q+7]) of that block. tb[(m*ntile+tt)*4+tp] = 16 * sum(hi+lo).
template <int NM, int PRO>
__device__ __forceinline__ void gemv_build_frags(const GemvParams& p, uint4* frag, float* tb, float* misc,
                                                 int ntile)
{
    const int tid = threadIdx.x, nth = blockDim.x;
    const int nblk = p.K >> 5;
    const float* src[NM];
    float rms[NM];
#pragma unroll
    for (int m = 0; m < NM; ++m)
    {
        src[m] = p.x + (size_t)m * p.lda;
        rms[m] = 1.0f;
    }
    if constexpr (PRO == PRO_EMBED_RMSNORM)
    {
        const uint32_t pos = p.state->pos;
        const uint32_t tok = pos < p.state->n_prompt ? p.prompt[pos] : p.state->next_token;
        src[0] = p.embedding + (size_t)tok * p.K;
        if (blockIdx.x == 0)
            for (int i = tid; i < p.K; i += nth)
                p.hidden_out[i] = src[0][i];
    }
    if constexpr (PRO != PRO_PLAIN)
    {
#pragma unroll
        for (int m = 0; m < NM; ++m)
        {
            float ss = 0.0f;
            for (int i = tid; i < p.K; i += nth)
            {
                float v = src[m][i];
                ss = fmaf(v, v, ss);
            }
            ss = block_sum(ss, misc);
            // src/rmsnorm.cpp:34
            rms[m] = 1.0f / sqrtf(__fadd_rn(__fdiv_rn(ss, (float)p.K), p.eps));
        }
    }
    const int nwords = NM * ntile * 16;
    for (int base = 0; base < nwords; base += nth)
    {
        const int wi = base + tid;
        const bool live = wi < nwords;
        const int m = live ? wi / (ntile * 16) : 0;
        const int rem = wi - m * ntile * 16;
        const int tt = rem >> 4, tl = rem & 15, tp = tl >> 2, q = tl & 3;
        const int blk = (p.kt0 + tt) * 4 + tp;
        float v[8];
        if (live && blk < nblk)
        {
            const int k0 = blk * 32 + q * 8;
            const float* xp = src[0];
#pragma unroll
            for (int mm = 1; mm < NM; ++mm)
                if (mm == m)
                    xp = src[mm];
            float r = rms[0];
#pragma unroll
            for (int mm = 1; mm < NM; ++mm)
                if (mm == m)
                    r = rms[mm];
#pragma unroll
            for (int c = 0; c < 8; ++c)
            {
                float xv = xp[k0 + c];
                if constexpr (PRO != PRO_PLAIN)
                    xv = __fmul_rn(__fmul_rn(xv, r), p.gain[k0 + c]); // src/rmsnorm.cpp:42-43
                v[c] = xv;
            }
        }
        else
        {
#pragma unroll
            for (int c = 0; c < 8; ++c)
                v[c] = 0.0f;
        }
        __nv_bfloat16 hi[8], lo[8];
        float tsum = 0.0f;
#pragma unroll
        for (int c = 0; c < 8; ++c)
        {
            hi[c] = __float2bfloat16_rn(v[c]);
            lo[c] = __float2bfloat16_rn(v[c] - __bfloat162float(hi[c]));
            tsum += __bfloat162float(hi[c]) + __bfloat162float(lo[c]);
        }
        if (live)
        {
            uint4* dst = frag + (((size_t)m * ntile + tt) * 4 + q) * 8 + 2 * tp;
            dst[0] = make_uint4(pack_bf16(hi[0], hi[4]), pack_bf16(hi[1], hi[5]), pack_bf16(hi[2], hi[6]),
                                pack_bf16(hi[3], hi[7]));
            dst[1] = make_uint4(pack_bf16(lo[0], lo[4]), pack_bf16(lo[1], lo[5]), pack_bf16(lo[2], lo[6]),
                                pack_bf16(lo[3], lo[7]));
        }
        tsum += __shfl_xor_sync(0xffffffffu, tsum, 1);
        tsum += __shfl_xor_sync(0xffffffffu, tsum, 2);
        if (live && q == 0)
            tb[((size_t)m * ntile + tt) * 4 + tp] = 16.0f * tsum;
    }
}

template <int NM, int PRO, int EPI, int SK, int R, int S>
__global__ void __launch_bounds__(GEMV_WARPS * 32) gemv_q4_kernel(const GemvParams p)
{
    static_assert(R * S == GEMV_WARPS, "R*S warps per CTA");
    extern __shared__ __align__(16) uint8_t smem[];
    const int ntile = p.kt1 - p.kt0;
    uint4* frag = reinterpret_cast<uint4*>(smem);
    float* tb = reinterpret_cast<float*>(smem + (size_t)NM * ntile * 512);
    float* red = tb + (size_t)NM * ntile * 4;
    float* misc = red + NM * S * R * 16;

    gemv_build_frags<NM, PRO>(p, frag, tb, misc, ntile);
    __syncthreads();

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, t = lane & 3;
    const int r = warp / S, s = warp - r * S;
    const int group = blockIdx.x * R + r;
    const int row0 = group * 16 + g, row1 = row0 + 8;
    const bool ok0 = row0 < p.N, ok1 = row1 < p.N;
    const int nblk = p.K >> 5;
    const uint8_t* w0p = p.w + (size_t)(ok0 ? row0 : 0) * (p.ldb >> 1);
    const uint8_t* w1p = p.w + (size_t)(ok1 ? row1 : 0) * (p.ldb >> 1);
    const uint16_t* s0p = p.s + (size_t)(ok0 ? row0 : 0) * (p.ldb >> 5);
    const uint16_t* s1p = p.s + (size_t)(ok1 ? row1 : 0) * (p.ldb >> 5);
    const int tA = (ntile * s) / S, tB = (ntile * (s + 1)) / S;
    const bool bact = (g >> 1) == t;
    const int la = 2 * t + (g & 1);

    float acc0[NM], acc1[NM];
#pragma unroll
    for (int m = 0; m < NM; ++m)
        acc0[m] = acc1[m] = 0.0f;

    if (group * 16 < p.N)
    {
        constexpr int PF = 4;
        uint4 W0[PF], W1[PF];
        float SC0[PF], SC1[PF];
#pragma unroll
        for (int i = 0; i < PF; ++i)
        {
            const int tt = tA + i;
            const int blk = (p.kt0 + tt) * 4 + t;
            const bool v = tt < tB && blk < nblk;
            W0[i] = (v && ok0) ? ldg_stream_v4(w0p + (size_t)blk * 16) : make_uint4(0, 0, 0, 0);
            W1[i] = (v && ok1) ? ldg_stream_v4(w1p + (size_t)blk * 16) : make_uint4(0, 0, 0, 0);
            SC0[i] = (v && ok0) ? decode_scale<SK>(ldg_u16(s0p + blk)) : 0.0f;
            SC1[i] = (v && ok1) ? decode_scale<SK>(ldg_u16(s1p + blk)) : 0.0f;
        }
        for (int tt0 = tA; tt0 < tB; tt0 += PF)
        {
#pragma unroll
            for (int i = 0; i < PF; ++i)
            {
                const int tt = tt0 + i;
                if (tt < tB)
                {
                    float d0[NM], d1[NM], d2[NM], d3[NM];
#pragma unroll
                    for (int m = 0; m < NM; ++m)
                        d0[m] = d1[m] = d2[m] = d3[m] = 0.0f;
#pragma unroll
                    for (int q = 0; q < 4; ++q)
                    {
                        const uint32_t wa = u4get(W0[i], q), wb = u4get(W1[i], q);
                        const uint32_t a0 = nib_e0(wa), a1 = nib_e0(wb), a2 = nib_e1(wa), a3 = nib_e1(wb);
                        const uint32_t c0 = nib_e2(wa), c1 = nib_e2(wb), c2 = nib_e3(wa), c3 = nib_e3(wb);
#pragma unroll
                        for (int m = 0; m < NM; ++m)
                        {
                            uint4 b = make_uint4(0, 0, 0, 0);
                            if (bact)
                                b = frag[(((size_t)m * ntile + tt) * 4 + q) * 8 + la];
                            mma_bf16_16816(d0[m], d1[m], d2[m], d3[m], a0, a1, a2, a3, b.x, b.y);
                            mma_bf16_16816(d0[m], d1[m], d2[m], d3[m], c0, c1, c2, c3, b.z, b.w);
                        }
                    }
#pragma unroll
                    for (int m = 0; m < NM; ++m)
                    {
                        const float tbv = tb[((size_t)m * ntile + tt) * 4 + t];
                        acc0[m] = fmaf(SC0[i], (d0[m] + d1[m]) - tbv, acc0[m]);
                        acc1[m] = fmaf(SC1[i], (d2[m] + d3[m]) - tbv, acc1[m]);
                    }
                    // refill this slot with the tile PF ahead
                    const int tn = tt + PF;
                    const int blk = (p.kt0 + tn) * 4 + t;
                    const bool v = tn < tB && blk < nblk;
                    W0[i] = (v && ok0) ? ldg_stream_v4(w0p + (size_t)blk * 16) : make_uint4(0, 0, 0, 0);
                    W1[i] = (v && ok1) ? ldg_stream_v4(w1p + (size_t)blk * 16) : make_uint4(0, 0, 0, 0);
                    SC0[i] = (v && ok0) ? decode_scale<SK>(ldg_u16(s0p + blk)) : 0.0f;
                    SC1[i] = (v && ok1) ? decode_scale<SK>(ldg_u16(s1p + blk)) : 0.0f;
                }
            }
        }
    }
#pragma unroll
    for (int m = 0; m < NM; ++m)
    {
        acc0[m] += __shfl_xor_sync(0xffffffffu, acc0[m], 1);
        acc0[m] += __shfl_xor_sync(0xffffffffu, acc0[m], 2);
        acc1[m] += __shfl_xor_sync(0xffffffffu, acc1[m], 1);
        acc1[m] += __shfl_xor_sync(0xffffffffu, acc1[m], 2);
        if (t == 0)
        {
            red[(m * S + s) * (R * 16) + r * 16 + g] = acc0[m];
            red[(m * S + s) * (R * 16) + r * 16 + g + 8] = acc1[m];
        }
    }
    __syncthreads();

    // ---------------- epilogues ----------------
    if constexpr (EPI == EPI_STORE || EPI == EPI_ACCUM || EPI == EPI_RESIDUAL)
    {
        for (int idx = tid; idx < NM * R * 16; idx += blockDim.x)
        {
            const int m = idx / (R * 16), rr = idx - m * R * 16;
            const int row = blockIdx.x * R * 16 + rr;
            if (row >= p.N)
                continue;
            float v = 0.0f;
            for (int ss = 0; ss < S; ++ss)
                v += red[(m * S + ss) * (R * 16) + rr];
            float* yp = p.y + (size_t)m * p.ldc + row;
            if constexpr (EPI == EPI_STORE)
                *yp = v;
            else
                *yp = v + *yp; // residual / K-chunk accumulation (src/transformer.cpp:214)
        }
    }
    else
    {
        for (int idx = tid; idx < R * 8; idx += blockDim.x)
        {
            const int rr = idx >> 3, jj = idx & 7;
            const int grp = blockIdx.x * R + rr;
            const int rbase = grp * 16;
            if (rbase >= p.N)
                continue;
            float v0 = 0.0f, v1 = 0.0f;
            for (int ss = 0; ss < S; ++ss)
            {
                v0 += red[ss * (R * 16) + rr * 16 + jj];
                v1 += red[ss * (R * 16) + rr * 16 + jj + 8];
            }
            if constexpr (EPI == EPI_SWIGLU)
            {
                // rows 8j..8j+7 of the gate and of up share one group (D6)
                p.act[grp * 8 + jj] = __fmul_rn(silu_f(v0), v1);
            }
            else
            {
                const int hd = p.head_dim, half = hd >> 1;
                const uint32_t pos = p.state->pos;
                if (pos >= (uint32_t)p.max_pos)
                {
                    if (jj == 0)
                        p.state->err = 1u;
                    continue;
                }
                const int page = p.page_table[pos / p.page_size];
                const int slot = pos % p.page_size;
                if (rbase < p.q_rows + p.kv_rows)
                {
                    const bool isq = rbase < p.q_rows;
                    const int rel = isq ? rbase : rbase - p.q_rows;
                    const int h = rel / hd, i = ((rel % hd) >> 4) * 8 + jj;
                    const float c = p.rope_cos[(size_t)pos * half + i];
                    const float sn = p.rope_sin[(size_t)pos * half + i];
                    // rotate-half (src/rope.cpp:53-54) at the absolute position (D3)
                    const float o0 = __fsub_rn(__fmul_rn(c, v0), __fmul_rn(sn, v1));
                    const float o1 = __fadd_rn(__fmul_rn(sn, v0), __fmul_rn(c, v1));
                    float* dst;
                    if (isq)
                        dst = p.qbuf + (size_t)h * hd;
                    else
                        dst = p.k_layer + (((size_t)page * p.n_kv + h) * p.page_size + slot) * hd;
                    dst[i] = o0;
                    dst[i + half] = o1;
                }
                else
                {
                    const int rel = rbase - p.q_rows - p.kv_rows;
                    const int h = rel / hd, d = rel % hd + jj;
                    float* dst = p.v_layer + (((size_t)page * p.n_kv + h) * p.page_size + slot) * hd;
                    dst[d] = v0;
                    dst[d + 8] = v1;
                }
            }
        }
    }
}

} // namespace aaedn_dev
