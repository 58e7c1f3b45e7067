// attention.cuh — split-K decode attention (one query token per head) over
// either a segment list (the reference API, src/attention.cpp:10-84) or a
// paged KV cache (the model path, D4/D5: causal MHA/GQA at the token's
// position).
//
// Grid (n_kv_heads, S): CTA (h, s) owns tokens [L*s/S, L*(s+1)/S) of kv head
// h and all G = n_heads/n_kv query heads that share it, so each K/V row is
// read from HBM once per step. Warp w of a CTA takes tokens w, w + 8, ... of
// that range, a batch at a time: each lane loads its 16-byte slices of the
// batch's K and V rows straight into registers (every load of the batch in
// flight at once), the q.k dots are finished with warp shuffles, and the
// softmax is carried online per warp (running max, sum and unnormalised V
// sum, rescaled when the max grows). The 8 warps, then the S splits (by the
// last CTA of each kv head), are merged in fixed order, so the result is
// deterministic. All arithmetic is fp32 with expf.
//
// In the model the K/V rows of earlier positions do not depend on the
// previous kernel: a CTA requests its first rows before waiting for it. The
// decode step's default is attn_decode_kernel (clusters, merge in
// distributed shared memory).
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
    float* part;        // [n_heads][S][pstride]: hd sums, max, sum
    int pstride;        // floats per partial result (0: hd + 2)
    unsigned* counters; // [n_kv], zero between launches
    int n_heads, n_kv, head_dim, S;
    float scale;
    const DecodeState* state; // MODE 1: L = pos + 1
    int len_static;           // MODE 0: L
    int max_len;              // bound on L (cache capacity)
    int max_tok;              // unused (kept for the launch interface)
    const int* page_table;
    int page_size;
    int nseg;
    uint32_t seg_start[ATTN_MAX_SEG];
    uint32_t seg_off[ATTN_MAX_SEG + 1]; // prefix sums of the lengths
    unsigned long long* trace; // per-CTA timeline of a traced step, or null
    // attn_decode_kernel over a batch of rows (grid.z = rows; null row_pos:
    // the one sequence at state->pos): row z is the token at position
    // row_pos[z] of sequence row_seq[z], whose page table starts at
    // page_table + row_seq[z] * pt_stride; q + z * ldq, out + z * ldo
    const int* row_pos;
    const int* row_seq;
    int pt_stride;
    size_t ldq, ldo;
    // warps a CTA of the clustered decode kernel for one query head per kv
    // head at head_dim <= 128 (10: more tokens in flight per split;
    // otherwise ATTN_WARPS)
    int warps;
};

// Shared memory: per-warp running max and sum [8][G] each, per-warp V sums
// [8][G][hd].
__host__ __device__ inline size_t attn_smem_bytes(int G, int hd, int /*max_tok*/)
{
    return ((size_t)2 * ATTN_WARPS * G + (size_t)ATTN_WARPS * G * hd) * 4;
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
        // a null page table is the identity (one sequence in pages 0, 1, ...)
        const int page = p.page_table ? p.page_table[t / p.page_size] : t / p.page_size;
        return (((size_t)page * p.n_kv + kvh) * p.page_size + (t % p.page_size)) * hd;
    }
}

// G: query heads per kv head; HDM: bound on head_dim (128 or 256).
// Registers: 64 per thread for MHA at head_dim <= 128 (4 CTAs per SM; a CTA
// also fits beside a GEMV CTA), more for the q and V-sum slices of several
// query heads.
constexpr int attn_min_blocks(int G, int HDM) { return (G == 1 && HDM == 128) ? 4 : (G * HDM >= 2048 ? 1 : 2); }

// Token range [t0, t1) of split `split` of S over L tokens.
__device__ __forceinline__ void attn_range(int L, int split, int S, int& t0, int& t1)
{
    t0 = (int)(((long long)L * split) / S);
    t1 = (int)(((long long)L * (split + 1)) / S);
}

template <int MODE>
__device__ __forceinline__ int attn_len(const AttnParams& p)
{
    int L = (MODE == 1) ? (int)p.state->pos + 1 : p.len_static;
    return L > p.max_len ? p.max_len : L;
}

// One work item, (kv head, split), on a group of ATTN_THREADS threads (tid =
// 0..255 within the group) that synchronise on named barrier bar_id: the
// split's partial result, and the merge of all S splits by the group that
// finishes a kv head last. asmem: attn_smem_bytes; s_last: one word of
// shared memory. PDLW: the item waits for the previous kernel itself, after
// it has requested its first batch of K/V rows (decode mode: every row but
// the current position's was written by earlier steps).
template <int MODE, int G, int HDM, bool PDLW = false>
__device__ __forceinline__ void attn_item(const AttnParams& p, int kvh, int split, int tid, float* asmem,
                                          unsigned* s_last, int bar_id)
{
    constexpr int NCH = HDM / 128;                         // float4 slices per lane
    constexpr int TB = (G == 1 && HDM == 128) ? 4 : 2;     // tokens per warp batch
    const int S = p.S;
    const int hd = p.head_dim, hd4 = hd >> 2;
    const int lane = tid & 31, warp = tid >> 5;
    int L = attn_len<MODE>(p);
    const int ps = p.pstride ? p.pstride : hd + 2;
    int t0, t1;
    attn_range(L, split, S, t0, t1);
    float* wm = asmem;                   // [8][G] running max per warp
    float* wl = wm + ATTN_WARPS * G;     // [8][G] running sum per warp
    float* wacc = wl + ATTN_WARPS * G;   // [8][G][hd]

    // batch loader: tokens tb0 + 8j, j < TB, K and V slices of this lane
    // (not token `skip`)
    float4 kr[TB][NCH], vr[TB][NCH];
    auto load_batch = [&](int tb0, int skip) {
#pragma unroll
        for (int j = 0; j < TB; ++j)
        {
            const int t = tb0 + ATTN_WARPS * j;
            const bool live = t < t1 && t != skip;
            const size_t ro = live ? attn_row<MODE>(p, t, kvh) : 0;
#pragma unroll
            for (int c = 0; c < NCH; ++c)
            {
                const int ch = lane + 32 * c;
                if (live && ch < hd4)
                {
                    kr[j][c] = __ldcg(reinterpret_cast<const float4*>(p.k + ro) + ch);
                    vr[j][c] = __ldcg(reinterpret_cast<const float4*>(p.v + ro) + ch);
                }
                else
                {
                    kr[j][c] = make_float4(0.f, 0.f, 0.f, 0.f);
                    vr[j][c] = make_float4(0.f, 0.f, 0.f, 0.f);
                }
            }
        }
    };
    // the first batch's rows are requested before q: their latencies overlap
    // (PDLW: before the wait for the kernel that writes q and row L - 1)
    const int tcur = (MODE == 1 && PDLW) ? L - 1 : -1;
    if (t0 + warp < t1)
        load_batch(t0 + warp, tcur);
    if constexpr (PDLW)
    {
        pdl_wait();
        if (tid == 0)
            trace_mark(p.trace, split * p.n_kv + kvh, 1);
        const int Lw = attn_len<MODE>(p);
        if (Lw != L)
        {
            // the position was read before the step before had finished
            // advancing it: take the range again with every row current
            L = Lw;
            attn_range(L, split, S, t0, t1);
            if (t0 + warp < t1)
                load_batch(t0 + warp, -1);
        }
        else
        {
#pragma unroll
            for (int j = 0; j < TB; ++j)
                if (t0 + warp + ATTN_WARPS * j == tcur && tcur < t1)
                {
                    const size_t ro = attn_row<MODE>(p, tcur, kvh);
#pragma unroll
                    for (int c = 0; c < NCH; ++c)
                    {
                        const int ch = lane + 32 * c;
                        if (ch < hd4)
                        {
                            kr[j][c] = __ldcg(reinterpret_cast<const float4*>(p.k + ro) + ch);
                            vr[j][c] = __ldcg(reinterpret_cast<const float4*>(p.v + ro) + ch);
                        }
                    }
                }
        }
    }
    // lane slices of q (scaled once: s = (q*scale).k would round differently,
    // so the scale is applied to the dot as src/attention.cpp:42 does)
    float4 qv[G][NCH];
#pragma unroll
    for (int gi = 0; gi < G; ++gi)
#pragma unroll
        for (int c = 0; c < NCH; ++c)
        {
            const int ch = lane + 32 * c;
            // L2 load: q is rewritten every layer (by other CTAs in the
            // persistent step kernel)
            qv[gi][c] = ch < hd4 ? __ldcg(reinterpret_cast<const float4*>(p.q + ((size_t)kvh * G + gi) * hd) + ch)
                                 : make_float4(0.f, 0.f, 0.f, 0.f);
        }
    float m[G], l[G];
    float4 acc[G][NCH];
#pragma unroll
    for (int gi = 0; gi < G; ++gi)
    {
        m[gi] = -INFINITY;
        l[gi] = 0.0f;
#pragma unroll
        for (int c = 0; c < NCH; ++c)
            acc[gi][c] = make_float4(0.f, 0.f, 0.f, 0.f);
    }

    for (int tb0 = t0 + warp; tb0 < t1; tb0 += ATTN_WARPS * TB)
    {
        if (tb0 != t0 + warp)
            load_batch(tb0, -1);
#pragma unroll
        for (int gi = 0; gi < G; ++gi)
        {
            float sj[TB];
#pragma unroll
            for (int j = 0; j < TB; ++j)
            {
                float d = 0.0f;
#pragma unroll
                for (int c = 0; c < NCH; ++c)
                {
                    d = fmaf(qv[gi][c].x, kr[j][c].x, d);
                    d = fmaf(qv[gi][c].y, kr[j][c].y, d);
                    d = fmaf(qv[gi][c].z, kr[j][c].z, d);
                    d = fmaf(qv[gi][c].w, kr[j][c].w, d);
                }
                sj[j] = d;
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1)
#pragma unroll
                for (int j = 0; j < TB; ++j)
                    sj[j] += __shfl_xor_sync(0xffffffffu, sj[j], o);
            float bm = -INFINITY;
#pragma unroll
            for (int j = 0; j < TB; ++j)
            {
                sj[j] = (tb0 + ATTN_WARPS * j < t1) ? sj[j] * p.scale : -INFINITY; // src/attention.cpp:42
                bm = fmaxf(bm, sj[j]);
            }
            const float mn = fmaxf(m[gi], bm);
            if (mn == -INFINITY)
                continue; // nothing live yet
            const float rs = (m[gi] == -INFINITY) ? 0.0f : expf(m[gi] - mn);
            m[gi] = mn;
            l[gi] *= rs;
#pragma unroll
            for (int c = 0; c < NCH; ++c)
            {
                acc[gi][c].x *= rs;
                acc[gi][c].y *= rs;
                acc[gi][c].z *= rs;
                acc[gi][c].w *= rs;
            }
#pragma unroll
            for (int j = 0; j < TB; ++j)
            {
                const float e = expf(sj[j] - mn); // 0 for dead slots
                l[gi] += e;
#pragma unroll
                for (int c = 0; c < NCH; ++c)
                {
                    acc[gi][c].x = fmaf(e, vr[j][c].x, acc[gi][c].x);
                    acc[gi][c].y = fmaf(e, vr[j][c].y, acc[gi][c].y);
                    acc[gi][c].z = fmaf(e, vr[j][c].z, acc[gi][c].z);
                    acc[gi][c].w = fmaf(e, vr[j][c].w, acc[gi][c].w);
                }
            }
        }
    }

    if (tid == 0)
        trace_mark(p.trace, split * p.n_kv + kvh, 2);
    // merge the 8 warps (fixed order) into this split's partial result
#pragma unroll
    for (int gi = 0; gi < G; ++gi)
    {
        if (lane == 0)
        {
            wm[warp * G + gi] = m[gi];
            wl[warp * G + gi] = l[gi];
        }
#pragma unroll
        for (int c = 0; c < NCH; ++c)
        {
            const int ch = lane + 32 * c;
            if (ch < hd4)
                reinterpret_cast<float4*>(wacc + ((size_t)warp * G + gi) * hd)[ch] = acc[gi][c];
        }
    }
    named_bar_sync(bar_id, ATTN_THREADS);
    for (int i = tid; i < G * hd; i += ATTN_THREADS)
    {
        const int gi = i / hd, d = i - gi * hd;
        float M = -INFINITY;
        for (int w = 0; w < ATTN_WARPS; ++w)
            M = fmaxf(M, wm[w * G + gi]);
        float o = 0.0f, den = 0.0f;
        for (int w = 0; w < ATTN_WARPS; ++w)
        {
            const float mw = wm[w * G + gi];
            const float f = (mw == -INFINITY) ? 0.0f : expf(mw - M);
            o = fmaf(wacc[((size_t)w * G + gi) * hd + d], f, o);
            den = fmaf(wl[w * G + gi], f, den);
        }
        const int h = kvh * G + gi;
        float* pp = p.part + ((size_t)h * S + split) * ps;
        pp[d] = o;
        if (d == 0)
        {
            pp[hd] = M;
            pp[hd + 1] = den;
        }
    }

    // last CTA of this kv head merges the S splits in order
    __threadfence();
    named_bar_sync(bar_id, ATTN_THREADS);
    if (tid == 0)
    {
        const unsigned prev = atomicAdd(&p.counters[kvh], 1u);
        *s_last = (prev == (unsigned)S - 1) ? 1u : 0u;
    }
    named_bar_sync(bar_id, ATTN_THREADS);
    if (!*s_last)
        return;
    __threadfence();
    for (int i = tid; i < G * hd; i += ATTN_THREADS)
    {
        const int gi = i / hd, d = i - gi * hd;
        const int h = kvh * G + gi;
        const float* pb = p.part + (size_t)h * S * ps;
        // splits in batches of SU with the loads unrolled (one L2 round trip
        // per batch, not per split); the sums still run in split order
        constexpr int SU = 8;
        float M = -INFINITY;
        for (int sb = 0; sb < S; sb += SU)
        {
            float mv[SU];
#pragma unroll
            for (int u = 0; u < SU; ++u)
                mv[u] = sb + u < S ? __ldcg(pb + (size_t)(sb + u) * ps + hd) : -INFINITY;
#pragma unroll
            for (int u = 0; u < SU; ++u)
                M = fmaxf(M, mv[u]);
        }
        float num = 0.0f, den = 0.0f;
        for (int sb = 0; sb < S; sb += SU)
        {
            float mv[SU], vv[SU], lv[SU];
#pragma unroll
            for (int u = 0; u < SU; ++u)
            {
                const bool live = sb + u < S;
                const float* pv = pb + (size_t)(sb + u) * ps;
                mv[u] = live ? __ldcg(pv + hd) : -INFINITY;
                vv[u] = live ? __ldcg(pv + d) : 0.0f;
                lv[u] = live ? __ldcg(pv + hd + 1) : 0.0f;
            }
#pragma unroll
            for (int u = 0; u < SU; ++u)
            {
                const float w = (mv[u] == -INFINITY) ? 0.0f : expf(mv[u] - M);
                num = fmaf(vv[u], w, num);
                den = fmaf(lv[u], w, den);
            }
        }
        p.out[(size_t)h * hd + d] = den > 0.0f ? num / den : 0.0f;
    }
    if (tid == 0)
        p.counters[kvh] = 0u;
}


// MODE 0: the reference API over a segment list. MODE 1: the model's decode
// step (splits merged through global memory by the last CTA of a kv head;
// the clustered kernel below is the default).
template <int MODE, int G, int HDM>
__global__ void __launch_bounds__(ATTN_THREADS, attn_min_blocks(G, HDM)) attn_split_kernel(const AttnParams p)
{
    extern __shared__ __align__(16) float asmem[];
    __shared__ unsigned s_last;
    pdl_launch_dependents();
    const int kvh = blockIdx.x, split = blockIdx.y, tid = threadIdx.x;
    const int lin = split * gridDim.x + kvh;
    if (tid == 0)
        trace_mark(p.trace, lin, 0);
    if constexpr (MODE == 1)
        attn_item<MODE, G, HDM, true>(p, kvh, split, tid, asmem, &s_last, 0); // waits for the previous kernel
    else
    {
        pdl_wait();
        attn_item<MODE, G, HDM>(p, kvh, split, tid, asmem, &s_last, 0);
    }
    if (tid == 0)
        trace_mark(p.trace, lin, 3);
}

// ---------------------------------------------------------------------------
// Decode attention as clusters: the S splits of one kv head are one cluster
// (grid (n_kv, S, rows), cluster (1, S)), CTA rank = split.
//   1. Split s takes tokens s, s + S, s + 2S, ...; warp w of its NW warps
//      (8, or 10 for MHA at head_dim <= 128: one batch of loads then covers
//      more context) the tokens s + S (w + NW j). The
//      rows of its first TB tokens (earlier positions) do not depend on the
//      kernel before, so each warp requests them (K and V straight into
//      registers) before waiting for the kernel that writes q and the
//      current K/V row: for the model's one sequence (identity page table)
//      those below the position read before the wait plus two (it may be
//      one step behind), for batched rows (launched after their positions
//      are written) those below the row's length. After the wait
//      the position bounds the tokens: rows at or past it are zeroed and
//      masked, the current row is requested again.
//   2. Online softmax per warp, as attn_item.
//   3. Each warp rescales its sums to the CTA's running max and the CTA adds
//      them in warp order: one partial (sums, max, denominator) per CTA,
//      which it writes into its slot of every cluster CTA's shared memory.
//   4. One cluster barrier; then every CTA merges a slice of the outputs over
//      the S partials from its own shared memory, in split order.
// ---------------------------------------------------------------------------

// MHA at head_dim <= 128: 64 registers, four CTAs of 8 warps (three of 10)
// per SM (a cluster then needs fewer free SMs of a GPC while the kernel
// before drains); wider groups keep their q and V sums for more heads in
// registers.
constexpr int attn_decode_min_blocks(int G, int HDM, int NW = ATTN_WARPS)
{
    return NW != ATTN_WARPS ? ((G == 1 && HDM == 128) ? 32 / NW : 1)
                            : (G == 1 && HDM == 128) ? 4 : (G * HDM >= 1024 ? 1 : 2);
}

// Shared memory: wm[NW][G], wl[NW][G], wacc[NW][G][hd] (NW warps a CTA),
// then the S partials [S][G][hd + 4] (sums, max, denominator; 16-byte rows).
__host__ __device__ inline size_t attn_decode_smem_bytes(int G, int hd, int S, int NW = ATTN_WARPS)
{
    return ((size_t)2 * NW * G + (size_t)NW * G * hd + (size_t)S * G * (hd + 4)) * 4;
}

__device__ __forceinline__ void st_dsmem_f32(uint32_t laddr, uint32_t rank, float v)
{
    uint32_t ra;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ra) : "r"(laddr), "r"(rank));
    asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(ra), "f"(v) : "memory");
}

template <int G, int HDM, bool CL = true, int NW = ATTN_WARPS>
__global__ void __launch_bounds__(NW * 32, attn_decode_min_blocks(G, HDM, NW)) attn_decode_kernel(const AttnParams p)
{
    constexpr int NCH = HDM / 128;                   // float4 slices per lane
    constexpr int TB = (G == 2 && NCH == 1) ? 8 : 4; // tokens per warp in flight
    extern __shared__ __align__(16) float asmem[];
    pdl_launch_dependents();
    const int kvh = blockIdx.x, split = blockIdx.y, S = (int)gridDim.y, z = blockIdx.z;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int hd = p.head_dim, hd4 = hd >> 2, ps = hd + 4;
    // this row's sequence: its page table (null: the identity)
    const int* pt = p.page_table && p.row_seq ? p.page_table + (size_t)p.row_seq[z] * p.pt_stride : p.page_table;
    auto row_of = [&](int t) -> size_t {
        const int page = pt ? pt[t / p.page_size] : t / p.page_size;
        return (((size_t)page * p.n_kv + kvh) * p.page_size + (t % p.page_size)) * hd;
    };
    auto tok = [&](int j) { return split + S * (warp + NW * j); }; // this warp's j-th token
    const float* qz = p.q + (size_t)z * p.ldq;
    float* outz = p.out + (size_t)z * p.ldo;
    float* wm = asmem;                         // [NW][G]
    float* wl = wm + NW * G;                   // [NW][G]
    float* wacc = wl + NW * G;                 // [NW][G][hd]
    float* parts = wacc + (size_t)NW * G * hd; // [S][G][hd + 4]
    const int lin = split * gridDim.x + kvh;
    if (tid == 0)
        trace_mark(p.trace, lin, 0);

    float4 kr[TB][NCH], vr[TB][NCH];
    auto load = [&](int jb, int lim) {
#pragma unroll
        for (int j = 0; j < TB; ++j)
        {
            const int t = tok(jb + j);
            const bool live = t < lim;
            const size_t ro = live ? row_of(t) : 0;
#pragma unroll
            for (int c = 0; c < NCH; ++c)
            {
                const int ch = lane + 32 * c;
                if (live && ch < hd4)
                {
                    kr[j][c] = __ldcg(reinterpret_cast<const float4*>(p.k + ro) + ch);
                    vr[j][c] = __ldcg(reinterpret_cast<const float4*>(p.v + ro) + ch);
                }
                else
                {
                    kr[j][c] = make_float4(0.f, 0.f, 0.f, 0.f);
                    vr[j][c] = make_float4(0.f, 0.f, 0.f, 0.f);
                }
            }
        }
    };
    // rows requested before the wait: below the row's length (batched rows are
    // launched after their positions are written), or, for the one sequence,
    // up to the position as it stands before the wait plus one: the kernel
    // that advances it may not have finished yet, and it moves by one a step
    // (the exact length bounds the tokens after the wait)
    const int lim0 = p.row_pos ? min(p.row_pos[z] + 1, p.max_len)
                               : min((int)*reinterpret_cast<const volatile uint32_t*>(&p.state->pos) + 2, p.max_len);
    load(0, lim0);
    pdl_wait();
    if (tid == 0)
        trace_mark(p.trace, lin, 1);
    float4 qv[G][NCH];
#pragma unroll
    for (int gi = 0; gi < G; ++gi)
#pragma unroll
        for (int c = 0; c < NCH; ++c)
        {
            const int ch = lane + 32 * c;
            qv[gi][c] = ch < hd4 ? __ldcg(reinterpret_cast<const float4*>(qz + ((size_t)kvh * G + gi) * hd) + ch)
                                 : make_float4(0.f, 0.f, 0.f, 0.f);
        }
    const int L = p.row_pos ? lim0 : attn_len<1>(p);
    // rows at or past L hold no token of this sequence (zero them: masked
    // weights times stale values must not give NaN); the current row L - 1
    // was written by the kernel before, and rows at or past the bound of the
    // requests before the wait (a position read more than a step behind)
    // were not requested
#pragma unroll
    for (int j = 0; j < TB; ++j)
    {
        const int t = tok(j);
        if (t >= L)
#pragma unroll
            for (int c = 0; c < NCH; ++c)
            {
                kr[j][c] = make_float4(0.f, 0.f, 0.f, 0.f);
                vr[j][c] = make_float4(0.f, 0.f, 0.f, 0.f);
            }
        else if (t == L - 1 || t >= lim0)
        {
            const size_t ro = row_of(t);
#pragma unroll
            for (int c = 0; c < NCH; ++c)
            {
                const int ch = lane + 32 * c;
                if (ch < hd4)
                {
                    kr[j][c] = __ldcg(reinterpret_cast<const float4*>(p.k + ro) + ch);
                    vr[j][c] = __ldcg(reinterpret_cast<const float4*>(p.v + ro) + ch);
                }
            }
        }
    }
    float m[G], l[G];
    float4 acc[G][NCH];
#pragma unroll
    for (int gi = 0; gi < G; ++gi)
    {
        m[gi] = -INFINITY;
        l[gi] = 0.0f;
#pragma unroll
        for (int c = 0; c < NCH; ++c)
            acc[gi][c] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    for (int jb = 0; tok(jb) < L; jb += TB)
    {
        if (jb)
            load(jb, L);
#pragma unroll
        for (int gi = 0; gi < G; ++gi)
        {
            float sj[TB];
#pragma unroll
            for (int j = 0; j < TB; ++j)
            {
                float d = 0.0f;
#pragma unroll
                for (int c = 0; c < NCH; ++c)
                {
                    d = fmaf(qv[gi][c].x, kr[j][c].x, d);
                    d = fmaf(qv[gi][c].y, kr[j][c].y, d);
                    d = fmaf(qv[gi][c].z, kr[j][c].z, d);
                    d = fmaf(qv[gi][c].w, kr[j][c].w, d);
                }
                sj[j] = d;
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1)
#pragma unroll
                for (int j = 0; j < TB; ++j)
                    sj[j] += __shfl_xor_sync(0xffffffffu, sj[j], o);
            float bm = -INFINITY;
#pragma unroll
            for (int j = 0; j < TB; ++j)
            {
                sj[j] = tok(jb + j) < L ? sj[j] * p.scale : -INFINITY; // src/attention.cpp:42
                bm = fmaxf(bm, sj[j]);
            }
            const float mn = fmaxf(m[gi], bm);
            if (mn == -INFINITY)
                continue;
            const float rs = (m[gi] == -INFINITY) ? 0.0f : expf(m[gi] - mn);
            m[gi] = mn;
            l[gi] *= rs;
#pragma unroll
            for (int c = 0; c < NCH; ++c)
            {
                acc[gi][c].x *= rs;
                acc[gi][c].y *= rs;
                acc[gi][c].z *= rs;
                acc[gi][c].w *= rs;
            }
#pragma unroll
            for (int j = 0; j < TB; ++j)
            {
                const float e = expf(sj[j] - mn); // 0 for masked slots
                l[gi] += e;
#pragma unroll
                for (int c = 0; c < NCH; ++c)
                {
                    acc[gi][c].x = fmaf(e, vr[j][c].x, acc[gi][c].x);
                    acc[gi][c].y = fmaf(e, vr[j][c].y, acc[gi][c].y);
                    acc[gi][c].z = fmaf(e, vr[j][c].z, acc[gi][c].z);
                    acc[gi][c].w = fmaf(e, vr[j][c].w, acc[gi][c].w);
                }
            }
        }
    }
    if (tid == 0)
        trace_mark(p.trace, lin, 2);

    // 3. the CTA's partial (warps rescaled to the CTA max, added in warp
    // order) into slot `split` of every CTA of the cluster
    if (lane == 0)
#pragma unroll
        for (int gi = 0; gi < G; ++gi)
            wm[warp * G + gi] = m[gi];
    __syncthreads();
#pragma unroll
    for (int gi = 0; gi < G; ++gi)
    {
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < NW; ++w)
            M = fmaxf(M, wm[w * G + gi]);
        const float f = (m[gi] == -INFINITY) ? 0.0f : expf(m[gi] - M);
        if (lane == 0)
            wl[warp * G + gi] = l[gi] * f;
#pragma unroll
        for (int c = 0; c < NCH; ++c)
        {
            const int ch = lane + 32 * c;
            if (ch < hd4)
                reinterpret_cast<float4*>(wacc + ((size_t)warp * G + gi) * hd)[ch] =
                    make_float4(acc[gi][c].x * f, acc[gi][c].y * f, acc[gi][c].z * f, acc[gi][c].w * f);
        }
    }
    __syncthreads();
    for (int i = tid; i < G * (hd + 2); i += NW * 32)
    {
        const int gi = i / (hd + 2), d = i - gi * (hd + 2);
        float v;
        if (d < hd)
        {
            v = 0.0f;
            for (int w = 0; w < NW; ++w)
                v += wacc[((size_t)w * G + gi) * hd + d];
        }
        else if (d == hd)
        {
            v = -INFINITY;
            for (int w = 0; w < NW; ++w)
                v = fmaxf(v, wm[w * G + gi]);
        }
        else
        {
            v = 0.0f;
            for (int w = 0; w < NW; ++w)
                v += wl[w * G + gi];
        }
        if constexpr (CL)
        {
            const uint32_t la = smem_addr(parts + ((size_t)split * G + gi) * ps + d);
            for (int r = 0; r < S; ++r)
                st_dsmem_f32(la, (uint32_t)r, v);
        }
        else
            p.part[(((size_t)z * p.n_heads + kvh * G + gi) * S + split) * ps + d] = v;
    }

    if constexpr (!CL)
    {
        // 4'. the last CTA of this (row, kv head) merges the S partials from
        // global memory, splits in order
        __shared__ unsigned s_last;
        __threadfence();
        __syncthreads();
        unsigned* ctr = p.counters + (size_t)z * p.n_kv + kvh;
        if (tid == 0)
            s_last = atomicAdd(ctr, 1u) == (unsigned)S - 1 ? 1u : 0u;
        __syncthreads();
        if (!s_last)
        {
            if (tid == 0)
                trace_mark(p.trace, lin, 3);
            return;
        }
        __threadfence();
        for (int i = tid; i < G * hd; i += NW * 32)
        {
            const int gi = i / hd, d = i - gi * hd;
            const float* pb = p.part + (((size_t)z * p.n_heads + kvh * G + gi) * S) * ps;
            // splits in batches of 8 with the loads of a batch issued together
            constexpr int SU = 8;
            float M = -INFINITY;
            for (int sb = 0; sb < S; sb += SU)
            {
                float mv[SU];
#pragma unroll
                for (int u = 0; u < SU; ++u)
                    mv[u] = sb + u < S ? __ldcg(pb + (size_t)(sb + u) * ps + hd) : -INFINITY;
#pragma unroll
                for (int u = 0; u < SU; ++u)
                    M = fmaxf(M, mv[u]);
            }
            float num = 0.0f, den = 0.0f;
            for (int sb = 0; sb < S; sb += SU)
            {
                float mv[SU], vv[SU], lv[SU];
#pragma unroll
                for (int u = 0; u < SU; ++u)
                {
                    const bool live = sb + u < S;
                    const float* pv = pb + (size_t)(sb + u) * ps;
                    mv[u] = live ? __ldcg(pv + hd) : -INFINITY;
                    vv[u] = live ? __ldcg(pv + d) : 0.0f;
                    lv[u] = live ? __ldcg(pv + hd + 1) : 0.0f;
                }
#pragma unroll
                for (int u = 0; u < SU; ++u)
                {
                    const float w = (mv[u] == -INFINITY) ? 0.0f : expf(mv[u] - M);
                    num = fmaf(vv[u], w, num);
                    den = fmaf(lv[u], w, den);
                }
            }
            outz[(size_t)(kvh * G + gi) * hd + d] = den > 0.0f ? num / den : 0.0f;
        }
        if (tid == 0)
        {
            *ctr = 0u;
            trace_mark(p.trace, lin, 3);
        }
        return;
    }

    // 4. one barrier (the partials written everywhere), then a slice of the
    // outputs per CTA from its own shared memory, splits in order
    cluster_sync_all();
    {
        const int n = G * hd, per = (n + S - 1) / S;
        for (int i = split * per + tid; i < min(n, (split + 1) * per); i += NW * 32)
        {
            const int gi = i / hd, d = i - gi * hd;
            float M = -INFINITY;
            for (int r = 0; r < S; ++r)
                M = fmaxf(M, parts[((size_t)r * G + gi) * ps + hd]);
            float num = 0.0f, den = 0.0f;
            for (int r = 0; r < S; ++r)
            {
                const float* pr = parts + ((size_t)r * G + gi) * ps;
                const float mr = pr[hd];
                const float w = (mr == -INFINITY) ? 0.0f : expf(mr - M);
                num = fmaf(pr[d], w, num);
                den = fmaf(pr[hd + 1], w, den);
            }
            outz[(size_t)(kvh * G + gi) * hd + d] = den > 0.0f ? num / den : 0.0f;
        }
    }
    if (tid == 0)
        trace_mark(p.trace, lin, 3);
}

} // namespace aaedn_dev

namespace aaedn_dev
{

template <int MODE, int G, int HDM>
inline cudaError_t attn_launch_one(const AttnParams& p, dim3 grid, size_t smem, cudaStream_t st, bool pdl)
{
    return launch_kernel(attn_split_kernel<MODE, G, HDM>, grid, dim3(ATTN_THREADS), smem, st, pdl, p);
}

// Shared memory of the clustered decode kernel.
inline size_t attn_cluster_smem_bytes(int G, int hd, int S) { return attn_decode_smem_bytes(G, hd, S); }

// Decode attention as clusters of grid.y CTAs (the splits of one kv head).
template <int G, int HDM, int NW = ATTN_WARPS>
inline cudaError_t attn_launch_cluster_one(const AttnParams& p, dim3 grid, cudaStream_t st, bool pdl)
{
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(NW * 32);
    cfg.dynamicSmemBytes = attn_decode_smem_bytes(G, p.head_dim, (int)grid.y, NW);
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = grid.y;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 2 : 1;
    return cudaLaunchKernelEx(&cfg, attn_decode_kernel<G, HDM, true, NW>, p);
}

inline int attn_launch_cluster(const AttnParams& p, dim3 grid, cudaStream_t st, bool pdl)
{
    const int G = p.n_heads / p.n_kv;
    const bool big = p.head_dim > 128;
    if ((int)grid.y != p.S || p.S > 16)
        return set_error(AAEDN_EINVAL, "clustered attention: %u CTAs per cluster for %d splits", grid.y, p.S);
    cudaError_t e;
    switch (G)
    {
    case 1:
        e = big               ? attn_launch_cluster_one<1, 256>(p, grid, st, pdl)
            : p.warps == 10   ? attn_launch_cluster_one<1, 128, 10>(p, grid, st, pdl)
                              : attn_launch_cluster_one<1, 128>(p, grid, st, pdl);
        break;
    case 2: e = big ? attn_launch_cluster_one<2, 256>(p, grid, st, pdl) : attn_launch_cluster_one<2, 128>(p, grid, st, pdl); break;
    case 4: e = big ? attn_launch_cluster_one<4, 256>(p, grid, st, pdl) : attn_launch_cluster_one<4, 128>(p, grid, st, pdl); break;
    case 8: e = big ? attn_launch_cluster_one<8, 256>(p, grid, st, pdl) : attn_launch_cluster_one<8, 128>(p, grid, st, pdl); break;
    default: return set_error(AAEDN_EUNSUPPORTED, "attention: %d query heads per kv head (1, 2, 4 or 8)", G);
    }
    if (e != cudaSuccess)
        return set_error(AAEDN_ECUDA, "launch of clustered attn_split_kernel failed: %s", cudaGetErrorString(e));
    count_launch();
    return AAEDN_OK;
}

// Decode attention with the splits merged through global memory by the
// last CTA of each (row, kv head) (p.part, p.counters).
template <int G, int HDM>
inline cudaError_t attn_launch_global_one(const AttnParams& p, dim3 grid, cudaStream_t st, bool pdl)
{
    return launch_kernel(attn_decode_kernel<G, HDM, false>, grid, dim3(ATTN_THREADS),
                         attn_decode_smem_bytes(G, p.head_dim, 0), st, pdl, p);
}

inline int attn_launch_global(const AttnParams& p, dim3 grid, cudaStream_t st, bool pdl)
{
    const int G = p.n_heads / p.n_kv;
    const bool big = p.head_dim > 128;
    if ((int)grid.y != p.S || p.S > 16)
        return set_error(AAEDN_EINVAL, "decode attention: %u splits for %d", grid.y, p.S);
    cudaError_t e;
    switch (G)
    {
    case 1: e = big ? attn_launch_global_one<1, 256>(p, grid, st, pdl) : attn_launch_global_one<1, 128>(p, grid, st, pdl); break;
    case 2: e = big ? attn_launch_global_one<2, 256>(p, grid, st, pdl) : attn_launch_global_one<2, 128>(p, grid, st, pdl); break;
    case 4: e = big ? attn_launch_global_one<4, 256>(p, grid, st, pdl) : attn_launch_global_one<4, 128>(p, grid, st, pdl); break;
    case 8: e = big ? attn_launch_global_one<8, 256>(p, grid, st, pdl) : attn_launch_global_one<8, 128>(p, grid, st, pdl); break;
    default: return set_error(AAEDN_EUNSUPPORTED, "attention: %d query heads per kv head (1, 2, 4 or 8)", G);
    }
    if (e != cudaSuccess)
        return set_error(AAEDN_ECUDA, "launch of attn_decode_kernel failed: %s", cudaGetErrorString(e));
    count_launch();
    return AAEDN_OK;
}

// Clusters of `S` CTAs that can be resident at once for head group G and
// head_dim hd (0: the variant can not run here).
template <int G, int HDM, int NW = ATTN_WARPS>
inline int attn_cluster_capacity_one(int S, int hd, int n_kv)
{
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(n_kv, S);
    cfg.blockDim = dim3(NW * 32);
    cfg.dynamicSmemBytes = attn_decode_smem_bytes(G, hd, S, NW);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = S;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, attn_decode_kernel<G, HDM, true, NW>, &cfg) != cudaSuccess)
    {
        cudaGetLastError();
        return 0;
    }
    return n;
}

inline int attn_cluster_capacity(int G, int hd, int S, int n_kv, int warps = ATTN_WARPS)
{
    const bool big = hd > 128;
    switch (G)
    {
    case 1:
        return big            ? attn_cluster_capacity_one<1, 256>(S, hd, n_kv)
               : warps == 10  ? attn_cluster_capacity_one<1, 128, 10>(S, hd, n_kv)
                              : attn_cluster_capacity_one<1, 128>(S, hd, n_kv);
    case 2: return big ? attn_cluster_capacity_one<2, 256>(S, hd, n_kv) : attn_cluster_capacity_one<2, 128>(S, hd, n_kv);
    case 4: return big ? attn_cluster_capacity_one<4, 256>(S, hd, n_kv) : attn_cluster_capacity_one<4, 128>(S, hd, n_kv);
    case 8: return big ? attn_cluster_capacity_one<8, 256>(S, hd, n_kv) : attn_cluster_capacity_one<8, 128>(S, hd, n_kv);
    default: return 0;
    }
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

// MODE 0: the API kernel; MODE 1: the model's decode kernels (clustered and
// global-merge variants).
template <int MODE, int G>
inline int attn_set_attrs_g()
{
    if constexpr (MODE == 0)
    {
        AAEDN_CUDA_TRY(cudaFuncSetAttribute(attn_split_kernel<0, G, 128>,
                                            cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
        AAEDN_CUDA_TRY(cudaFuncSetAttribute(attn_split_kernel<0, G, 256>,
                                            cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
    }
    else
    {
        // clusters of up to 16 CTAs
        AAEDN_CUDA_TRY(cudaFuncSetAttribute(attn_decode_kernel<G, 128>,
                                            cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
        AAEDN_CUDA_TRY(cudaFuncSetAttribute(attn_decode_kernel<G, 256>,
                                            cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
        AAEDN_CUDA_TRY(cudaFuncSetAttribute(attn_decode_kernel<G, 128>,
                                            cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
        AAEDN_CUDA_TRY(cudaFuncSetAttribute(attn_decode_kernel<G, 256>,
                                            cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
        AAEDN_CUDA_TRY(cudaFuncSetAttribute(attn_decode_kernel<G, 128, false>,
                                            cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
        AAEDN_CUDA_TRY(cudaFuncSetAttribute(attn_decode_kernel<G, 256, false>,
                                            cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
    }
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
