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
//    two codes, then c with one bf16x2 subtraction (exact: 4-bit integers are
//    exact in bf16), so no bias has to be removed after the accumulation
//    (that would lose the low bits of blocks whose large activations meet
//    zero codes);
//  * the tensor core (mma.sync m16n8k16 bf16 -> fp32) is used as the dot
//    product engine: A = 16 weight rows x 16 codes; the activation is split
//    into three bf16 parts x = hi + mid + lo (24 significant bits, as many
//    as fp32 carries), the B columns of one mma are 4 quant blocks x (hi,
//    mid) and those of a second mma 4 blocks x (lo, 0), so each lane's fp32
//    accumulators hold the per-(row, block) partial sums its own block
//    needs;
//  * the per-block epilogue applies the block scale in fp32;
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
    // tensor parallel: the rows of this rank's partial sum go to its slot of
    // its own receive buffer; the kernel's last CTA pushes the slot to every
    // other rank through peer memory
    EPI_TP_PUSH = 5,
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

constexpr int TP_MAX = 8;

// The peer-visible regions of the tensor-parallel ranks (CUDA IPC): each
// holds partials [2][dim] floats, flag words (one per writer rank, 16 bytes
// apart) and argmax slots.
struct TpComm
{
    // receive buffers of every rank (own included): recv[p] + (src * 2 +
    // buf) * dim holds source rank src's partial `buf` (0: o, 1: down)
    float* recv[TP_MAX];
    unsigned* flags[TP_MAX]; // flag words of every rank: flags[p][4 * w] = epoch written by w
    float2* best[TP_MAX];    // argmax slots of every rank: best[p][w] = (value, index) of w
    unsigned* my_flags;      // == flags[rank]
    int rank, size, dim;
};

constexpr uint64_t TP_WAIT_LIMIT_NS = 2000000000ull; // 2 s



// Waits (bounded) until every rank's flag word in this rank's array shows
// epoch E. On success a system-scope fence follows the flag reads, so the
// caller's later loads (and those of threads it releases through a barrier)
// see what the peers wrote before raising their flags (tp_signal fences at
// system scope before its flag stores).
__device__ __forceinline__ bool tp_wait_flags(const TpComm& c, unsigned E, DecodeState* st)
{
    const uint64_t t0 = globaltimer_ns();
    volatile uint32_t* err = &st->err;
    for (int w = 0; w < c.size; ++w)
    {
        volatile unsigned* f = c.my_flags + 4 * w;
        while (*f < E)
        {
            // a wait that already ran out in this step (sticky error): the
            // later ones give up at once instead of waiting their full limit
            if (*err != 0u || globaltimer_ns() - t0 > TP_WAIT_LIMIT_NS)
            {
                *err = 4u;
                return false;
            }
            __nanosleep(32);
        }
    }
    __threadfence_system();
    return true;
}

// Raise this rank's flag for epoch E in every rank's flag array (itself
// included), after its earlier writes are visible to the peers.
__device__ __forceinline__ void tp_signal(const TpComm& c, unsigned E)
{
    __threadfence_system();
    for (int p = 0; p < c.size; ++p)
    {
        volatile unsigned* f = c.flags[p] + 4 * c.rank;
        *f = E;
    }
}

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
    int l2_hint; // stream the weights with the L2 evict-first policy
    unsigned long long* trace; // per-CTA timeline of a traced step (tiled kernel), or null
    int stages;                // ring stages of the tiled kernel (0: GT_STAGES)
    // tensor parallel (zero otherwise): a partial-writing GEMV (tp_sig)
    // stores its rows in partial buffer tp_buf and raises epoch *tp_epoch +
    // tp_sig_phase + 1 in every rank once its last CTA is done (tp_counter:
    // last-CTA count)
    TpComm tpc;
    const unsigned* tp_epoch;
    unsigned* tp_counter;
    int tp_buf, tp_sig, tp_sig_phase;
    // scales can be staged as aligned u32 pairs (even scales per row, 4-byte
    // aligned array)
    bool scale_pairs;
    // N % 16 == 0 and K % 128 == 0: no padding rows or blocks anywhere
    bool full_shape;
};

constexpr int GEMV_WARPS = 8;
constexpr int GEMV_STAGES = 6; // per-thread cp.async ring depth (tiles)

// Activation fragments of one 128-code tile: 4 k-steps x 16 lane slots
// (8 for the (hi, mid) mma, 8 for the (lo, 0) mma) x 16 B.
constexpr int GEMV_FRAG_TILE_BYTES = 1024;

// Dynamic shared memory of one CTA: the cp.async ring (6 stages x 256
// threads x 40 B), the activation fragments (and one zero tile), block
// biases, two reduction buffers.
inline size_t gemv_smem_bytes(int nm, int ntile)
{
    return (size_t)GEMV_STAGES * GEMV_WARPS * 32 * 40 + (size_t)(nm * ntile + 1) * GEMV_FRAG_TILE_BYTES +
           (size_t)nm * ntile * 16 +
           (size_t)2 * nm * GEMV_WARPS * 16 * 4 + 64 * 4;
}

__device__ __forceinline__ uint32_t u4get(const uint4& v, int q)
{
    return q == 0 ? v.x : (q == 1 ? v.y : (q == 2 ? v.z : v.w));
}

// Sum over the first NTH threads (warps 0..NTH/32-1, named barrier 1);
// every one of them receives the result. scratch >= NTH/32 floats.
template <int NTH>
__device__ __forceinline__ float group_sum(float v, float* scratch)
{
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    v = warp_sum(v);
    named_bar_sync(1, NTH);
    if (lane == 0)
        scratch[warp] = v;
    named_bar_sync(1, NTH);
    float t = 0.0f;
    for (int i = 0; i < NTH / 32; ++i) // fixed order: deterministic
        t += scratch[i];
    named_bar_sync(1, NTH);
    return t;
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
// frag[((m*ntile + tt)*4 + q)*16 + la] holds, for lane slot la = 2*tp + p
// (block tp of the tile; p = 0: hi, 1: mid) and la = 8 + 2*tp + p (p = 0:
// lo, 1: zero), the 4 bf16x2 registers of mmas 2q and 2q+1: (x[8q+0],x[8q+4]),
// (x[8q+1],x[8q+5]), (x[8q+2],x[8q+6]), (x[8q+3],x[8q+7]) of that part of the
// block.
template <int NM, int PRO, int NTH = GEMV_WARPS * 32>
__device__ __forceinline__ void gemv_build_frags(const GemvParams& p, uint4* frag, float* tb, float* misc,
                                                 int ntile)
{
    const int tid = threadIdx.x, nth = NTH;
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
            const float4* s4 = reinterpret_cast<const float4*>(src[m]);
            for (int i = tid; i < (p.K >> 2); i += nth)
            {
                const float4 v = s4[i];
                ss = fmaf(v.x, v.x, ss);
                ss = fmaf(v.y, v.y, ss);
                ss = fmaf(v.z, v.z, ss);
                ss = fmaf(v.w, v.w, ss);
            }
            ss = group_sum<NTH>(ss, misc);
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
            if ((reinterpret_cast<uintptr_t>(xp + k0) & 15) == 0)
            {
                const float4 a = *reinterpret_cast<const float4*>(xp + k0);
                const float4 b = *reinterpret_cast<const float4*>(xp + k0 + 4);
                v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
            }
            else
            {
#pragma unroll
                for (int c = 0; c < 8; ++c)
                    v[c] = xp[k0 + c];
            }
            if constexpr (PRO != PRO_PLAIN)
            {
                const float4 ga = *reinterpret_cast<const float4*>(p.gain + k0);
                const float4 gb = *reinterpret_cast<const float4*>(p.gain + k0 + 4);
                const float gv[8] = {ga.x, ga.y, ga.z, ga.w, gb.x, gb.y, gb.z, gb.w};
#pragma unroll
                for (int c = 0; c < 8; ++c)
                    v[c] = __fmul_rn(__fmul_rn(v[c], r), gv[c]); // src/rmsnorm.cpp:42-43
            }
        }
        else
        {
#pragma unroll
            for (int c = 0; c < 8; ++c)
                v[c] = 0.0f;
        }
        // x = hi + mid + lo: each part the bf16 rounding of what the parts
        // before it leave (the differences are exact in fp32)
        __nv_bfloat16 hi[8], mid[8], lo[8];
#pragma unroll
        for (int c = 0; c < 8; ++c)
        {
            hi[c] = __float2bfloat16_rn(v[c]);
            const float r1 = v[c] - __bfloat162float(hi[c]);
            mid[c] = __float2bfloat16_rn(r1);
            lo[c] = __float2bfloat16_rn(r1 - __bfloat162float(mid[c]));
        }
        if (live)
        {
            uint4* dst = frag + (((size_t)m * ntile + tt) * 4 + q) * 16 + 2 * tp;
            dst[0] = make_uint4(pack_bf16(hi[0], hi[4]), pack_bf16(hi[1], hi[5]), pack_bf16(hi[2], hi[6]),
                                pack_bf16(hi[3], hi[7]));
            dst[1] = make_uint4(pack_bf16(mid[0], mid[4]), pack_bf16(mid[1], mid[5]), pack_bf16(mid[2], mid[6]),
                                pack_bf16(mid[3], mid[7]));
            dst[8] = make_uint4(pack_bf16(lo[0], lo[4]), pack_bf16(lo[1], lo[5]), pack_bf16(lo[2], lo[6]),
                                pack_bf16(lo[3], lo[7]));
            dst[9] = make_uint4(0u, 0u, 0u, 0u);
        }
    }
}

// Epilogue of one 16-row group on one warp: sums the S K-split partial
// sums of each row in fixed order, then stores / accumulates / adds the
// residual, or pairs rows (8j + r, 8j + r + 8) for SwiGLU and for RoPE +
// the KV-cache append.
// Epilogue inputs staged in shared memory before a CTA's first group (so
// the warp that runs an epilogue does not wait on global loads while the
// other warps need it to release ring stages): the residual rows of the
// CTA's groups (resid[gl * 16 + r], gl = the CTA's group number), or the RoPE
// row of the position (cos[half], sin[half]) and the cache page.
struct EpiCache
{
    const float* resid;
    const float* cos;
    const float* sin;
    int page;
};

template <int NM, int EPI, int S = GEMV_WARPS>
__device__ __forceinline__ void gemv_epilogue(const GemvParams& p, const float* rb, int group, int lane,
                                              float post = 1.0f, const EpiCache* ec = nullptr, int gl = 0)
{
    if constexpr (EPI == EPI_STORE || EPI == EPI_ACCUM || EPI == EPI_RESIDUAL || EPI == EPI_TP_PUSH)
    {
        for (int idx = lane; idx < NM * 16; idx += 32)
        {
            const int m = idx >> 4, rr = idx & 15;
            const int row = group * 16 + rr;
            if (row >= p.N)
                continue;
            float v = 0.0f;
            for (int ss = 0; ss < S; ++ss)
                v += rb[(m * S + ss) * 16 + rr];
            v *= post; // the RMSNorm factor of the warp-built operand (1: exact no-op)
            if constexpr (EPI == EPI_TP_PUSH)
            {
                // this rank's slot of its own receive buffer (the kernel's last
                // CTA then copies the whole partial to the other ranks)
                p.tpc.recv[p.tpc.rank][((size_t)p.tpc.rank * 2 + p.tp_buf) * p.tpc.dim + row] = v;
                continue;
            }
            float* yp = p.y + (size_t)m * p.ldc + row;
            if constexpr (EPI == EPI_STORE)
                *yp = v;
            else // residual / K-chunk accumulation (src/transformer.cpp:214)
                *yp = v + (ec ? ec->resid[gl * 16 + rr] : __ldcg(yp));
        }
    }
    else
    {
        const int jj = lane;
        const int rbase = group * 16;
        if (jj >= 8 || rbase >= p.N)
            return;
        float v0 = 0.0f, v1 = 0.0f;
        for (int ss = 0; ss < S; ++ss)
        {
            v0 += rb[ss * 16 + jj];
            v1 += rb[ss * 16 + jj + 8];
        }
        v0 *= post;
        v1 *= post;
        if constexpr (EPI == EPI_SWIGLU)
        {
            // rows 8j..8j+7 of the gate and of up share one group (D6)
            p.act[group * 8 + jj] = __fmul_rn(silu_f(v0), v1);
        }
        else
        {
            const int hd = p.head_dim, half = hd >> 1;
            const uint32_t pos = p.state->pos;
            if (pos >= (uint32_t)p.max_pos)
            {
                if (jj == 0)
                    p.state->err = 1u;
                return;
            }
            const int page = ec ? ec->page : p.page_table[pos / p.page_size];
            const int slot = pos % p.page_size;
            if (rbase < p.q_rows + p.kv_rows)
            {
                const bool isq = rbase < p.q_rows;
                const int rel = isq ? rbase : rbase - p.q_rows;
                const int h = rel / hd, i = ((rel % hd) >> 4) * 8 + jj;
                const float c = ec ? ec->cos[i] : p.rope_cos[(size_t)pos * half + i];
                const float sn = ec ? ec->sin[i] : p.rope_sin[(size_t)pos * half + i];
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

// The main loop for full shapes (N a multiple of 16, K a multiple of 128,
// scales staged in pairs): every copy and every fragment read is
// unconditional and all shared-memory addresses are 32-bit.
template <int NM, int EPI, int SK, typename Issue>
__device__ __forceinline__ void gemv_lean_loop(const GemvParams& p, uint4* stw, uint32_t* sts, uint4* frag, float* tb,
                                               float* red, int my_groups, int tA, int tB, int ntile, Issue& issue)
{
    constexpr int D = GEMV_STAGES;
    constexpr int NT = GEMV_WARPS * 32;
    constexpr int S = GEMV_WARPS;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, t = lane & 3;
    const bool bact = (g >> 1) == t;
    const int la = 2 * t + (g & 1);
    // scale pair half: blk & 1 == t & 1 for every tile of this thread
    const uint32_t hsel = (t & 1) ? 0x3232u : 0x1010u;
    const uint32_t w_base = smem_addr(stw) + (uint32_t)tid * 32;
    const uint32_t s_base = smem_addr(sts) + (uint32_t)tid * 8;
    // inactive lanes read their (zero) B operand from the fragment area of a
    // tile past the end, which the prologue zero-fills
    const uint32_t f_base = smem_addr(frag) + (uint32_t)la * 16;
    const uint32_t f_zero = smem_addr(frag) + (uint32_t)NM * ntile * GEMV_FRAG_TILE_BYTES;
    uint32_t c_off_w = 0, c_off_s = 0;
    for (int gl = 0; gl < my_groups; ++gl)
    {
        const int group = blockIdx.x + gl * gridDim.x;
        float acc0[NM], acc1[NM];
#pragma unroll
        for (int m = 0; m < NM; ++m)
            acc0[m] = acc1[m] = 0.0f;
        uint32_t fa = bact ? f_base + (uint32_t)tA * GEMV_FRAG_TILE_BYTES : f_zero;
        const uint32_t fstep = bact ? (uint32_t)GEMV_FRAG_TILE_BYTES : 0u;
        const uint32_t mstride = bact ? (uint32_t)ntile * GEMV_FRAG_TILE_BYTES : 0u;
        for (int tt = tA; tt < tB; ++tt, fa += fstep)
        {
            cp_async_wait<D - 2>();
            const uint4 wa4 = lds128(w_base + c_off_w);
            const uint4 wb4 = lds128(w_base + c_off_w + 16);
            const uint32_t pa = lds32(s_base + c_off_s), pb = lds32(s_base + c_off_s + 4);
            const float sc0 = decode_scale<SK>((uint16_t)__byte_perm(pa, 0, hsel));
            const float sc1 = decode_scale<SK>((uint16_t)__byte_perm(pb, 0, hsel));
            c_off_w = (c_off_w == (D - 1) * NT * 32) ? 0u : c_off_w + NT * 32;
            c_off_s = (c_off_s == (D - 1) * NT * 8) ? 0u : c_off_s + NT * 8;
            issue();

            float d0[NM], d1[NM], d2[NM], d3[NM], e0[NM], e1[NM], e2[NM], e3[NM];
#pragma unroll
            for (int m = 0; m < NM; ++m)
                d0[m] = d1[m] = d2[m] = d3[m] = e0[m] = e1[m] = e2[m] = e3[m] = 0.0f;
#pragma unroll
            for (int q = 0; q < 4; ++q)
            {
                const uint32_t wa = u4get(wa4, q), wb = u4get(wb4, q);
                const uint32_t a0 = unbias16(nib_e0(wa)), a1 = unbias16(nib_e0(wb));
                const uint32_t a2 = unbias16(nib_e1(wa)), a3 = unbias16(nib_e1(wb));
                const uint32_t c0 = unbias16(nib_e2(wa)), c1 = unbias16(nib_e2(wb));
                const uint32_t c2 = unbias16(nib_e3(wa)), c3 = unbias16(nib_e3(wb));
#pragma unroll
                for (int m = 0; m < NM; ++m)
                {
                    const uint32_t fq = fa + (uint32_t)m * mstride + (uint32_t)(q * 256);
                    const uint4 b = lds128(fq), bl = lds128(fq + 128);
                    mma_bf16_16816(d0[m], d1[m], d2[m], d3[m], a0, a1, a2, a3, b.x, b.y);
                    mma_bf16_16816(d0[m], d1[m], d2[m], d3[m], c0, c1, c2, c3, b.z, b.w);
                    mma_bf16_16816(e0[m], e1[m], e2[m], e3[m], a0, a1, a2, a3, bl.x, bl.y);
                    mma_bf16_16816(e0[m], e1[m], e2[m], e3[m], c0, c1, c2, c3, bl.z, bl.w);
                }
            }
#pragma unroll
            for (int m = 0; m < NM; ++m)
            {
                // columns 2t / 2t+1 of the first mma: (hi, mid); column 2t of the second: lo
                acc0[m] = fmaf(sc0, (d0[m] + d1[m]) + e0[m], acc0[m]);
                acc1[m] = fmaf(sc1, (d2[m] + d3[m]) + e2[m], acc1[m]);
            }
        }
        float* rb = red + (size_t)(gl & 1) * NM * S * 16;
#pragma unroll
        for (int m = 0; m < NM; ++m)
        {
            acc0[m] += __shfl_xor_sync(0xffffffffu, acc0[m], 1);
            acc0[m] += __shfl_xor_sync(0xffffffffu, acc0[m], 2);
            acc1[m] += __shfl_xor_sync(0xffffffffu, acc1[m], 1);
            acc1[m] += __shfl_xor_sync(0xffffffffu, acc1[m], 2);
            if (t == 0)
            {
                rb[(m * S + warp) * 16 + g] = acc0[m];
                rb[(m * S + warp) * 16 + g + 8] = acc1[m];
            }
        }
        __syncthreads();
        if (warp == (gl & (GEMV_WARPS - 1)))
            gemv_epilogue<NM, EPI>(p, rb, group, lane);
    }
}

// One CTA of 8 warps per SM (persistent): the CTA takes row groups
// blockIdx.x, blockIdx.x + gridDim.x, ... and its 8 warps split K of each
// group. Every thread streams its 16-byte code words (rows g and g+8) and
// scale pairs through a private cp.async ring that runs straight through group
// boundaries. A CTA needs well under half of an SM, so the next kernel of a
// decode step (launched as a programmatic dependent) becomes resident at once
// and fills its own ring while this one computes.
template <int NM, int PRO, int EPI, int SK, bool FULL = false>
__global__ void __launch_bounds__(GEMV_WARPS * 32, 2) gemv_q4_kernel(const GemvParams p)
{
    constexpr int D = GEMV_STAGES;
    constexpr int NT = GEMV_WARPS * 32;
    constexpr int S = GEMV_WARPS; // K splits of a group
    extern __shared__ __align__(16) uint8_t smem[];
    const int ntile = p.kt1 - p.kt0;
    // [D][NT][2] code words of rows g and g+8, [D][NT][2] scale pairs, then
    // the activation fragments, block biases, two reduction buffers.
    uint4* stw = reinterpret_cast<uint4*>(smem);
    uint32_t* sts = reinterpret_cast<uint32_t*>(smem + (size_t)D * NT * 32);
    uint4* frag = reinterpret_cast<uint4*>(smem + (size_t)D * NT * 40);
    // one zero tile after the fragments: the B operand of inactive lanes
    float* tb = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(frag) +
                                         (size_t)(NM * ntile + 1) * GEMV_FRAG_TILE_BYTES);
    float* red = tb + (size_t)NM * ntile * 4; // [2][NM][S][16]
    float* misc = red + 2 * NM * S * 16;

    // the next kernel in the stream may start its own weight prefetch now
    pdl_launch_dependents();

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, t = lane & 3;
    const int s = warp;
    const int nblk = p.K >> 5;
    const int n_groups = (p.N + 15) >> 4;
    const int my_groups = blockIdx.x < n_groups ? (n_groups - 1 - blockIdx.x) / gridDim.x + 1 : 0;
    const int tA = (ntile * s) / S, tB = (ntile * (s + 1)) / S;
    const bool bact = (g >> 1) == t;
    const int la = 2 * t + (g & 1);
    const bool pairs = p.scale_pairs;
    const size_t wrow = p.ldb >> 1, srow = p.ldb >> 5;
    const size_t gstride_w = (size_t)16 * gridDim.x * wrow, gstride_s = (size_t)16 * gridDim.x * srow;
    const int blk0 = p.kt0 * 4 + t; // block of tile 0 of this thread
    const int shift = (blk0 & 1) * 16; // which half of a scale pair (constant per thread)

    // ---- issue cursor: walks (group, tile) pairs in order, no divisions
    int i_tt = tA, i_left = (tB > tA) ? my_groups : 0, i_slot = 0;
    int i_row0 = blockIdx.x * 16 + g;
    const uint8_t* i_w0 = p.w + (size_t)i_row0 * wrow + (size_t)blk0 * 16;
    const uint8_t* i_w1 = i_w0 + 8 * wrow;
    const uint16_t* i_s0 = p.s + (size_t)i_row0 * srow + (blk0 & ~1);
    const uint16_t* i_s1 = i_s0 + 8 * srow;
    const uint32_t ring_w = smem_addr(stw) + (uint32_t)tid * 32;
    const uint32_t ring_s = smem_addr(sts) + (uint32_t)tid * 8;
    constexpr bool full = FULL;
    auto issue = [&]() {
        if (i_left > 0)
        {
            const bool vb = full || blk0 + 4 * i_tt < nblk;
            const bool v0 = full || (vb && i_row0 < p.N), v1 = full || (vb && i_row0 + 8 < p.N);
            const size_t off = (size_t)i_tt * 64;
            const uint32_t dw = ring_w + (uint32_t)i_slot * (NT * 32);
            asm volatile("cp.async.cg.shared.global.L2::256B [%0], [%1], 16, %2;" ::"r"(dw),
                         "l"(v0 ? i_w0 + off : p.w), "r"(v0 ? 16u : 0u)
                         : "memory");
            asm volatile("cp.async.cg.shared.global.L2::256B [%0], [%1], 16, %2;" ::"r"(dw + 16),
                         "l"(v1 ? i_w1 + off : p.w), "r"(v1 ? 16u : 0u)
                         : "memory");
            if (pairs)
            {
                const uint32_t ds = ring_s + (uint32_t)i_slot * (NT * 8);
                asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(ds),
                             "l"(v0 ? i_s0 + 4 * i_tt : p.s), "r"(v0 ? 4u : 0u)
                             : "memory");
                asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(ds + 4),
                             "l"(v1 ? i_s1 + 4 * i_tt : p.s), "r"(v1 ? 4u : 0u)
                             : "memory");
            }
            if (++i_tt == tB)
            {
                i_tt = tA;
                --i_left;
                i_row0 += 16 * gridDim.x;
                i_w0 += gstride_w;
                i_w1 += gstride_w;
                i_s0 += gstride_s;
                i_s1 += gstride_s;
            }
        }
        i_slot = (i_slot + 1 == D) ? 0 : i_slot + 1;
        cp_async_commit();
    };

    // The weights do not depend on the activations: the first D-1 items are
    // requested before waiting for the previous kernel and before the
    // activation prologue, so their HBM latency overlaps both.
#pragma unroll
    for (int i = 0; i < D - 1; ++i)
        issue();

    pdl_wait();
    gemv_build_frags<NM, PRO>(p, frag, tb, misc, ntile);
    if (tid < GEMV_FRAG_TILE_BYTES / 16)
        frag[(size_t)NM * ntile * (GEMV_FRAG_TILE_BYTES / 16) + tid] = make_uint4(0, 0, 0, 0);
    __syncthreads();

    if (FULL)
    {
        gemv_lean_loop<NM, EPI, SK>(p, stw, sts, frag, tb, red, my_groups, tA, tB, ntile, issue);
        cp_async_wait<0>();
        return;
    }

    int c_slot = 0;
    int row0 = blockIdx.x * 16 + g;
    for (int gl = 0; gl < my_groups; ++gl, row0 += 16 * gridDim.x)
    {
        const int group = blockIdx.x + gl * gridDim.x;
        const bool ok0 = row0 < p.N, ok1 = row0 + 8 < p.N;
        float acc0[NM], acc1[NM];
#pragma unroll
        for (int m = 0; m < NM; ++m)
            acc0[m] = acc1[m] = 0.0f;
        constexpr int FT = GEMV_FRAG_TILE_BYTES / 16; // uint4 per tile
        const uint4* fb = frag + (size_t)tA * FT + la;
        for (int tt = tA; tt < tB; ++tt, fb += FT)
        {
            cp_async_wait<D - 2>(); // this thread's copies of this item have landed
            const uint4* wsl = stw + (size_t)c_slot * NT * 2 + (size_t)tid * 2;
            const uint4 wa4 = wsl[0], wb4 = wsl[1];
            float sc0, sc1;
            if (pairs)
            {
                const uint32_t* ssl = sts + (size_t)c_slot * NT * 2 + (size_t)tid * 2;
                sc0 = decode_scale<SK>((uint16_t)(ssl[0] >> shift));
                sc1 = decode_scale<SK>((uint16_t)(ssl[1] >> shift));
            }
            else
            {
                const int blk = blk0 + 4 * tt;
                const bool v = blk < nblk;
                sc0 = (v && ok0) ? decode_scale<SK>(ldg_u16(p.s + (size_t)row0 * srow + blk)) : 0.0f;
                sc1 = (v && ok1) ? decode_scale<SK>(ldg_u16(p.s + (size_t)(row0 + 8) * srow + blk)) : 0.0f;
            }
            c_slot = (c_slot + 1 == D) ? 0 : c_slot + 1;
            // refill the slot consumed in the previous iteration
            issue();

            float d0[NM], d1[NM], d2[NM], d3[NM], e0[NM], e1[NM], e2[NM], e3[NM];
#pragma unroll
            for (int m = 0; m < NM; ++m)
                d0[m] = d1[m] = d2[m] = d3[m] = e0[m] = e1[m] = e2[m] = e3[m] = 0.0f;
#pragma unroll
            for (int q = 0; q < 4; ++q)
            {
                const uint32_t wa = u4get(wa4, q), wb = u4get(wb4, q);
                const uint32_t a0 = unbias16(nib_e0(wa)), a1 = unbias16(nib_e0(wb));
                const uint32_t a2 = unbias16(nib_e1(wa)), a3 = unbias16(nib_e1(wb));
                const uint32_t c0 = unbias16(nib_e2(wa)), c1 = unbias16(nib_e2(wb));
                const uint32_t c2 = unbias16(nib_e3(wa)), c3 = unbias16(nib_e3(wb));
#pragma unroll
                for (int m = 0; m < NM; ++m)
                {
                    uint4 b = make_uint4(0, 0, 0, 0), bl = b;
                    if (bact)
                    {
                        b = fb[(size_t)m * ntile * FT + q * 16];
                        bl = fb[(size_t)m * ntile * FT + q * 16 + 8];
                    }
                    mma_bf16_16816(d0[m], d1[m], d2[m], d3[m], a0, a1, a2, a3, b.x, b.y);
                    mma_bf16_16816(d0[m], d1[m], d2[m], d3[m], c0, c1, c2, c3, b.z, b.w);
                    mma_bf16_16816(e0[m], e1[m], e2[m], e3[m], a0, a1, a2, a3, bl.x, bl.y);
                    mma_bf16_16816(e0[m], e1[m], e2[m], e3[m], c0, c1, c2, c3, bl.z, bl.w);
                }
            }
#pragma unroll
            for (int m = 0; m < NM; ++m)
            {
                acc0[m] = fmaf(sc0, (d0[m] + d1[m]) + e0[m], acc0[m]);
                acc1[m] = fmaf(sc1, (d2[m] + d3[m]) + e2[m], acc1[m]);
            }
        }
        float* rb = red + (size_t)(gl & 1) * NM * S * 16;
#pragma unroll
        for (int m = 0; m < NM; ++m)
        {
            acc0[m] += __shfl_xor_sync(0xffffffffu, acc0[m], 1);
            acc0[m] += __shfl_xor_sync(0xffffffffu, acc0[m], 2);
            acc1[m] += __shfl_xor_sync(0xffffffffu, acc1[m], 1);
            acc1[m] += __shfl_xor_sync(0xffffffffu, acc1[m], 2);
            if (t == 0)
            {
                rb[(m * S + s) * 16 + g] = acc0[m];
                rb[(m * S + s) * 16 + g + 8] = acc1[m];
            }
        }
        __syncthreads(); // the reduction buffer of the other parity is free again
        // epilogue of this group on the warp gl % 8 (the others stream on)
        if (warp == (gl & (GEMV_WARPS - 1)))
            gemv_epilogue<NM, EPI>(p, rb, group, lane);
    }
    cp_async_wait<0>(); // nothing of this thread stays in flight past here
}

} // namespace aaedn_dev
