// gemv_tiled.cuh — the decode dequant-GEMV over tile-major ("tiled") weights.
//
// The model repacks every quantized matrix once at load time. The blocks and
// scales are the reference's (32 codes = 16 bytes, one fp16 scale per block);
// only their order in memory changes, so that everything one CTA step needs
// is one contiguous run:
//   matrix = row groups of 16 rows, in order
//   group  = chunks of up to 32 tiles (a tile = 128 codes of each of the 16
//            rows = 1 KB of codes), the last chunk of a group may be short
//   chunk  = codes [tile i][half h][lane l][16 B] then scales [tile i][half
//            h][lane l] (u16), where lane l = 4g + t holds block 4i + t of row
//            g + 8h: exactly the A-fragment order of the mma.
// A row group's K range is one linear stream, so one bulk (TMA) copy moves a
// whole chunk (up to 36 KB) and DRAM sees long sequential bursts; a warp's
// 16-byte reads of a tile cover 512 consecutive shared-memory bytes (no bank
// conflicts).
//
// CTA: one producer warp (bulk copies into a 4-stage ring, mbarriers) + 16
// consumer warps; consumer warp w computes tiles w and w + 16 of every chunk,
// interleaved as four independent accumulator chains.
#pragma once

#include "gemv_q4.cuh"

namespace aaedn_dev
{

constexpr uint64_t GEMV_WAIT_LIMIT_NS = 2000000000ull; // 2 s: bound of every mbarrier wait

constexpr int GT_CONSUMERS = 16;
constexpr int GT_THREADS = (GT_CONSUMERS + 1) * 32;
constexpr int GT_STAGES = 4;     // ring stages of the persistent step kernel; the
                                 // decode GEMV takes what its shared memory allows
constexpr int GT_MAX_STAGES = 8;
constexpr int GT_CHUNK_TILES = 32; // two tiles per consumer warp
constexpr int GT_TILE_BYTES = 1024 + 128; // codes + scales of one tile (16 rows x 128 codes)
constexpr int GT_STAGE_BYTES = GT_CHUNK_TILES * GT_TILE_BYTES; // 36 KB
// Group reductions in flight (integer engine): RB buffers of [16 warps][16
// rows] partial sums, each with an arrival counter; the warp that completes a
// group runs its epilogue, the others go on (no CTA-wide barrier per group).
constexpr int GT_RB = 8;
constexpr int GT_RED_BYTES = GT_RB * GT_CONSUMERS * 16 * 4 + GT_RB * 4 + 96;
// Shared memory for the staged epilogue inputs (EpiCache): 2048 floats.
constexpr int GT_ECACHE_FLOATS = 2048;

// Bytes of a repacked matrix (same as the row-major codes + scales).
inline size_t tiled_bytes(size_t N, size_t K) { return N * K / 2 + N * K / 32 * 2; }

// Repacks row-major codes/scales ([N][K], K % 128 == 0, N % 16 == 0).
void repack_tiled(const uint8_t* codes, const uint16_t* scales, size_t N, size_t K, uint8_t* out);

// ---------------------------------------------------------------------------
// Integer dot-product engine.
//
// The activation x (after the prologue) is rescaled to y = x * 127 / max|x|
// and written as four signed base-128 digits, y = d0 + d1/128 + d2/128^2 +
// d3/128^3 + e with |e| <= 2^-22, so that a block's dot product with the
// 4-bit codes is four exact integer sums, computed by the u8 x s8 mma. The
// codes stay as they are in memory: the low nibble of every byte (even
// element) is fed as c, the high nibble in place as 16*c, and the odd
// elements' digits are those of y/16 to match. One k32 mma covers 8 codes of
// each of 4 blocks (one block per lane t of a quad); its 8 columns are (block,
// digit) pairs, so one mma yields digits (0,1) and a second digits (2,3),
// and four k-steps complete the tile's 4 blocks with nothing rounded.
// ---------------------------------------------------------------------------

inline size_t gemv_tiled_i8_smem_bytes(int ntile, int stages = GT_STAGES)
{
    return (size_t)stages * GT_STAGE_BYTES + (size_t)stages * 16 + (size_t)ntile * (512 + 16) + GT_RED_BYTES +
           64 * 4 + GT_ECACHE_FLOATS * 4;
}

// The most ring stages (<= GT_MAX_STAGES) whose shared memory fits `budget`.
inline int gemv_tiled_stages(int ntile, size_t budget)
{
    int s = GT_MAX_STAGES;
    while (s > 2 && gemv_tiled_i8_smem_bytes(ntile, s) > budget)
        --s;
    return s;
}

// The shared-memory ring of a tiled GEMV CTA: stage i at ring + i * 36 KB,
// full[i] / empty[i] mbarriers. Chunks are numbered in the order the producer
// issues them (q); chunk q sits in stage q % GT_STAGES, use q / GT_STAGES.
struct TiledRing
{
    uint32_t ring, full, empty; // shared-memory addresses
    uint32_t ns;                // stages
};

// Producer warp: issues, for every row group this CTA owns (cta, cta + ncta,
// ...), its chunks of the tile-major matrix w ([N/16][K/128 tiles]). Returns
// false if a wait for a free stage ran out (the caller drains and stops).
__device__ __forceinline__ bool tiled_produce(const uint8_t* w, int N, int K, const TiledRing& r, uint32_t& q,
                                              int cta, int ncta, int lane, unsigned long long* wait_cycles = nullptr,
                                              bool hint = false)
{
    constexpr int CT = GT_CHUNK_TILES;
    const uint32_t NS = r.ns;
    const int ntile = K >> 7, nchunk = (ntile + CT - 1) / CT, n_groups = N >> 4;
    const size_t group_bytes = (size_t)ntile * GT_TILE_BYTES;
    // stage and use of chunk q, advanced without a division per chunk
    uint32_t stage = q % NS, use = q / NS;
    for (int group = cta; group < n_groups; group += ncta)
    {
        const uint8_t* gsrc = w + (size_t)group * group_bytes;
        for (int c = 0; c < nchunk; ++c, ++q, (++stage == NS) ? (stage = 0, ++use) : 0u)
        {
            const int tiles = (c + 1) * CT <= ntile ? CT : ntile - c * CT;
            const long long c0 = wait_cycles ? clock64() : 0;
            if (use > 0 && !mbar_wait_bounded(r.empty + 8 * stage, (use - 1) & 1, GEMV_WAIT_LIMIT_NS))
                return false;
            if (wait_cycles)
                *wait_cycles += (unsigned long long)(clock64() - c0);
            if (lane == 0)
            {
                const uint32_t bytes = (uint32_t)tiles * GT_TILE_BYTES;
                mbar_arrive_expect_tx(r.full + 8 * stage, bytes);
                if (hint)
                    bulk_g2s_hint(r.ring + stage * GT_STAGE_BYTES, gsrc + (size_t)c * CT * GT_TILE_BYTES, bytes,
                                  r.full + 8 * stage, l2_evict_first_policy());
                else
                    bulk_g2s(r.ring + stage * GT_STAGE_BYTES, gsrc + (size_t)c * CT * GT_TILE_BYTES, bytes,
                             r.full + 8 * stage);
            }
            __syncwarp();
        }
    }
    return true;
}

// Producer warp before exit: every issued chunk (q of them) has landed.
__device__ __forceinline__ void tiled_drain(const TiledRing& r, uint32_t q)
{
    const uint32_t NS = r.ns;
    for (uint32_t k = (q > NS ? q - NS : 0); k < q; ++k)
        mbar_wait_bounded(r.full + 8 * (k % NS), (k / NS) & 1, GEMV_WAIT_LIMIT_NS);
}

// ---------------------------------------------------------------------------
// Warp-built operand (the persistent step kernel's GEMVs).
//
// Consumer warp w only ever reads tiles w and w + 16 of every chunk, so it
// builds exactly those tiles' B operands itself: no CTA-wide barrier between
// the activation and the first weight chunk. The activation is scaled per
// 32-element block (y = x * 127 / max|x| over the block, unit = max / (127 *
// 128) kept in bscale), so the digits need no reduction over the whole
// vector; the RMSNorm factor is a scalar applied after the dot product
// (W (r * (x o g)) = r * W (x o g)), from the per-warp sums of squares in
// wss, summed in fixed order by the warp that runs each group's epilogue.
// ---------------------------------------------------------------------------

// Builds this warp's tiles: frag slots, bscale[tile * 4 + block] and (NORM)
// wss[warp]. zero16: a 16-byte zero in shared memory (B of inactive lanes).
template <int PRO>
__device__ __forceinline__ void warp_build_i8(const GemvParams& p, uint4* frag, float* bscale, float* wss,
                                              unsigned long long* pass_a_cycles = nullptr,
                                              volatile unsigned* cta_flag = nullptr)
{
    const long long c_start = pass_a_cycles ? clock64() : 0;
    constexpr bool NORM = PRO == PRO_RMSNORM || PRO == PRO_EMBED_RMSNORM || PRO == PRO_TP_RMSNORM;
    constexpr int NC = GT_CONSUMERS, CT = GT_CHUNK_TILES;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    // the CTA's warps start on different tiles (CTA c shifts by c): 148 CTAs
    // do not all ask L2 for the same lines of x at the same moment
    const int wv = (warp + (int)blockIdx.x) & (NC - 1);
    const int ntile = p.K >> 7, nchunk = (ntile + CT - 1) / CT;
    const float* src = p.x;
    if constexpr (PRO == PRO_EMBED_RMSNORM)
    {
        const uint32_t pos = p.state->pos;
        const uint32_t tok = pos < p.state->n_prompt ? p.prompt[pos] : p.state->next_token;
        src = p.embedding + (size_t)tok * p.K;
    }
    if constexpr (PRO == PRO_TP_RMSNORM)
    {
        // the ranks' partials of the previous GEMV are in this rank's receive
        // buffer once their flags show its epoch: warp 0 waits on the flags,
        // the other warps on warp 0 (bounded waits; a timeout is reported
        // through DecodeState::err)
        if (lane == 0)
        {
            const unsigned E = *p.tp_epoch + (unsigned)p.tp_wait_phase + 1u;
            if (warp == 0)
            {
                tp_wait_flags(p.tpc, E, p.state);
                __threadfence_system();
                *cta_flag = E;
            }
            else
            {
                const uint64_t t0 = globaltimer_ns();
                while (*cta_flag < E && globaltimer_ns() - t0 < TP_WAIT_LIMIT_NS)
                    __nanosleep(32);
                __threadfence_system();
            }
        }
        __syncwarp();
    }
    const int item = lane & 15, tb = item >> 2, s = item & 3;
    float ss = 0.0f;
    // pass A: every chunk's loads issued back to back (one L2 round trip for
    // the whole operand); the raw x*g values are parked in their frag slots
#pragma unroll 4
    for (int c = 0; c < nchunk; ++c)
    {
        const int tiles = (c + 1) * CT <= ntile ? CT : ntile - c * CT;
        const int ti = wv + NC * (lane >> 4); // lanes 0-15: tile wv, 16-31: tile wv + 16
        const bool live = ti < tiles;
        const int tile = c * CT + ti;
        const int k0 = tile * 128 + tb * 32 + s * 8;
        float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        if (live)
        {
            float4 a, b;
            if constexpr (PRO == PRO_ATTN_COMBINE)
            {
                // elements k0..k0+7 of head h: the merge of its S split
                // results, in split order, as the attention kernel's own merge
                constexpr int SU = 16;
                const int hd = p.head_dim, h = k0 / hd, d0 = k0 - h * hd, S = p.attn_S, ps = p.attn_pstride;
                const float* pb = p.attn_part + (size_t)h * S * ps;
                float num[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f}, den = 0.0f;
                // splits in batches of SU, loads unrolled (one L2 round trip
                // per batch); the sums run in split order
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
                for (int sb = 0; sb < S; sb += SU)
                {
                    float ms[SU], ls[SU];
#pragma unroll
                    for (int u = 0; u < SU; ++u)
                    {
                        const float2 ml = sb + u < S
                                              ? __ldcg(reinterpret_cast<const float2*>(pb + (size_t)(sb + u) * ps + hd))
                                              : make_float2(-INFINITY, 0.0f);
                        ms[u] = ml.x;
                        ls[u] = ml.y;
                    }
#pragma unroll
                    for (int u = 0; u < SU; ++u)
                        if (sb + u < S)
                        {
                            const float* pv = pb + (size_t)(sb + u) * ps + d0;
                            const float4 va = __ldcg(reinterpret_cast<const float4*>(pv));
                            const float4 vb = __ldcg(reinterpret_cast<const float4*>(pv + 4));
                            const float w = (ms[u] == -INFINITY) ? 0.0f : expf(ms[u] - M);
                            num[0] = fmaf(va.x, w, num[0]);
                            num[1] = fmaf(va.y, w, num[1]);
                            num[2] = fmaf(va.z, w, num[2]);
                            num[3] = fmaf(va.w, w, num[3]);
                            num[4] = fmaf(vb.x, w, num[4]);
                            num[5] = fmaf(vb.y, w, num[5]);
                            num[6] = fmaf(vb.z, w, num[6]);
                            num[7] = fmaf(vb.w, w, num[7]);
                            den = fmaf(ls[u], w, den);
                        }
                }
#pragma unroll
                for (int cc = 0; cc < 8; ++cc)
                    v[cc] = den > 0.0f ? num[cc] / den : 0.0f;
            }
            else
            {
                // L2 loads: in the persistent step kernel x was written by
                // other CTAs after this SM may have cached an older copy in L1
                a = __ldcg(reinterpret_cast<const float4*>(src + k0));
                b = __ldcg(reinterpret_cast<const float4*>(src + k0 + 4));
                if constexpr (PRO == PRO_TP_RMSNORM)
                {
                    // residual + the ranks' partials (this rank's receive
                    // buffer), summed in rank order: the same value on every
                    // rank
                    float4 sa = make_float4(0.f, 0.f, 0.f, 0.f), sb = sa;
                    const float* rb = p.tpc.recv[p.tpc.rank] + (size_t)p.tp_buf * p.tpc.dim + k0;
                    for (int w = 0; w < p.tpc.size; ++w)
                    {
                        const float* pw = rb + (size_t)w * 2 * p.tpc.dim;
                        const float4 pa = __ldcg(reinterpret_cast<const float4*>(pw));
                        const float4 pb = __ldcg(reinterpret_cast<const float4*>(pw + 4));
                        sa.x += pa.x, sa.y += pa.y, sa.z += pa.z, sa.w += pa.w;
                        sb.x += pb.x, sb.y += pb.y, sb.z += pb.z, sb.w += pb.w;
                    }
                    a = make_float4(a.x + sa.x, a.y + sa.y, a.z + sa.z, a.w + sa.w);
                    b = make_float4(b.x + sb.x, b.y + sb.y, b.z + sb.z, b.w + sb.w);
                }
                v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
                if constexpr (PRO == PRO_EMBED_RMSNORM || PRO == PRO_TP_RMSNORM)
                    if (blockIdx.x == 0)
                    {
                        *reinterpret_cast<float4*>(p.hidden_out + k0) = a;
                        *reinterpret_cast<float4*>(p.hidden_out + k0 + 4) = b;
                    }
            }
            if constexpr (NORM)
            {
                const float4 ga = __ldg(reinterpret_cast<const float4*>(p.gain + k0));
                const float4 gb = __ldg(reinterpret_cast<const float4*>(p.gain + k0 + 4));
                const float gv[8] = {ga.x, ga.y, ga.z, ga.w, gb.x, gb.y, gb.z, gb.w};
#pragma unroll
                for (int cc = 0; cc < 8; ++cc)
                {
                    ss = fmaf(v[cc], v[cc], ss);
                    v[cc] = __fmul_rn(v[cc], gv[cc]); // src/rmsnorm.cpp:42-43 without the 1/rms
                }
            }
        }
        if (live)
        {
            float4* park = reinterpret_cast<float4*>(frag + ((size_t)tile * 4 + s) * 8 + 2 * tb);
            park[0] = make_float4(v[0], v[1], v[2], v[3]);
            park[1] = make_float4(v[4], v[5], v[6], v[7]);
        }
    }
    __syncwarp();
    if (pass_a_cycles)
        *pass_a_cycles += (unsigned long long)(clock64() - c_start);
    // pass B: block maxima and digits, in place
    for (int c = 0; c < nchunk; ++c)
    {
        const int tiles = (c + 1) * CT <= ntile ? CT : ntile - c * CT;
        const int ti = wv + NC * (lane >> 4);
        const bool live = ti < tiles;
        const int tile = c * CT + ti;
        float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        if (live)
        {
            const float4* park = reinterpret_cast<const float4*>(frag + ((size_t)tile * 4 + s) * 8 + 2 * tb);
            const float4 a = park[0], b = park[1];
            v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
        }
        // block max over the 4 lanes of the block (items s = 0..3); a
        // non-finite value makes the block's unit NaN (so its outputs are)
        float mx = 0.0f;
        bool fin = true;
#pragma unroll
        for (int cc = 0; cc < 8; ++cc)
        {
            const float a8 = fabsf(v[cc]);
            fin = fin && (a8 <= 3.0e38f);
            mx = fmaxf(mx, a8);
        }
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
        const unsigned bad = __ballot_sync(0xffffffffu, !fin);
        const bool bbad = ((bad >> (lane & ~3)) & 0xFu) != 0;
        const float inv = (mx > 0.0f && !bbad) ? 127.0f / mx : 0.0f;
        if (live)
        {
            // balanced base-128 digits of Y = round(y * 2^21) (odd elements:
            // of y/16, so Y = round(y * 2^17)), exact integer arithmetic:
            // Y = d0 2^21 + d1 2^14 + d2 2^7 + d3, d0 in [-127, 127], the
            // others in [-64, 64]
            int dg[8][4];
#pragma unroll
            for (int cc = 0; cc < 8; ++cc)
            {
                const float y = __fmul_rn(v[cc], inv);
                const int Y = __float2int_rn(y * ((cc & 1) ? 131072.0f : 2097152.0f));
                const int d0 = (Y + (1 << 20)) >> 21;
                const int r0 = Y - (d0 << 21);
                const int d1 = (r0 + (1 << 13)) >> 14;
                const int r1 = r0 - (d1 << 14);
                const int d2 = (r1 + 64) >> 7;
                dg[cc][0] = d0;
                dg[cc][1] = d1;
                dg[cc][2] = d2;
                dg[cc][3] = r1 - (d2 << 7);
            }
            // one word = the bytes of one digit of elements e, e+2, e+4, e+6
            auto pack = [&](int e, int k) {
                const uint32_t lo = __byte_perm((uint32_t)dg[e][k], (uint32_t)dg[e + 2][k], 0x0040);
                const uint32_t hi = __byte_perm((uint32_t)dg[e + 4][k], (uint32_t)dg[e + 6][k], 0x0040);
                return __byte_perm(lo, hi, 0x5410);
            };
            const uint32_t w0[4] = {pack(0, 0), pack(1, 0), pack(0, 2), pack(1, 2)};
            const uint32_t w1[4] = {pack(0, 1), pack(1, 1), pack(0, 3), pack(1, 3)};
            uint4* dst = frag + ((size_t)tile * 4 + s) * 8 + 2 * tb;
            dst[0] = make_uint4(w0[0], w0[1], w0[2], w0[3]);
            dst[1] = make_uint4(w1[0], w1[1], w1[2], w1[3]);
            if (s == 0)
                bscale[tile * 4 + tb] = bbad ? __int_as_float(0x7fc00000) : mx / (127.0f * 128.0f);
        }
    }
    if constexpr (NORM)
    {
        ss = warp_sum(ss);
        if (lane == 0)
            wss[warp] = ss;
    }
    __syncwarp();
}

// Consumer warps of one GEMV with warp-built operands (warp_build_i8 first,
// in the same warp). zero16: shared address of 16 zero bytes.
template <int PRO, int EPI>
__device__ __forceinline__ bool tiled_wb_consume(const GemvParams& p, const TiledRing& r, uint32_t& q,
                                                 const uint4* frag, const float* bscale, const float* wss,
                                                 uint32_t zero16, float* red, float* ecache, int cta, int ncta,
                                                 volatile int& s_abort, unsigned long long* wait_cycles = nullptr)
{
    constexpr bool NORM = PRO == PRO_RMSNORM || PRO == PRO_EMBED_RMSNORM || PRO == PRO_TP_RMSNORM;
    const uint32_t NS = r.ns;
    constexpr int NC = GT_CONSUMERS;
    constexpr int NCT = NC * 32;
    constexpr int CT = GT_CHUNK_TILES;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int wv = (warp + (int)blockIdx.x) & (NC - 1); // the tiles warp_build_i8 gave this warp
    const int ntile = p.K >> 7, nchunk = (ntile + CT - 1) / CT, n_groups = p.N >> 4;
    const int g = lane >> 2, t = lane & 3;
    const bool bact = (g >> 1) == t;
    const uint32_t f_base = bact ? smem_addr(frag) + (uint32_t)g * 16 : zero16;
    const uint32_t f_step = bact ? 512u : 0u;
    const uint32_t f_sstep = bact ? 128u : 0u;
    const uint32_t bs_base = smem_addr(bscale) + (uint32_t)t * 4;
    // epilogue inputs into shared memory (read by whichever warp completes a
    // group; every warp has stored its share before its first arrival)
    EpiCache ec{};
    const EpiCache* ecp = nullptr;
    if constexpr (EPI == EPI_RESIDUAL)
    {
        const int my_groups = cta < n_groups ? (n_groups - 1 - cta) / ncta + 1 : 0;
        if (my_groups * 16 <= GT_ECACHE_FLOATS)
        {
            for (int i = tid; i < my_groups * 16; i += NCT)
                ecache[i] = __ldcg(p.y + (size_t)(cta + (i >> 4) * ncta) * 16 + (i & 15));
            ec.resid = ecache;
            ecp = &ec;
        }
    }
    else if constexpr (EPI == EPI_QKV_ROPE)
    {
        const int half = p.head_dim >> 1;
        const uint32_t pos = p.state->pos;
        if (half <= GT_ECACHE_FLOATS / 2 - 1 && pos < (uint32_t)p.max_pos)
        {
            for (int i = tid; i < half; i += NCT)
            {
                ecache[i] = __ldg(p.rope_cos + (size_t)pos * half + i);
                ecache[GT_ECACHE_FLOATS / 2 + i] = __ldg(p.rope_sin + (size_t)pos * half + i);
            }
            ec.cos = ecache;
            ec.sin = ecache + GT_ECACHE_FLOATS / 2;
            ec.page = __ldg(p.page_table + pos / p.page_size);
            ecp = &ec;
        }
    }
    bool ok = true;
    int gl = 0;
    uint32_t stage = q % NS, phase = (q / NS) & 1; // advanced without a division per chunk
    for (int group = cta; group < n_groups; group += ncta, ++gl)
    {
        float acc0 = 0.0f, acc1 = 0.0f;
        for (int c = 0; c < nchunk && ok; ++c, ++q, (++stage == NS) ? (stage = 0, phase ^= 1u) : 0u)
        {
            const int tiles = (c + 1) * CT <= ntile ? CT : ntile - c * CT;
            const long long c0 = wait_cycles ? clock64() : 0;
            if (!mbar_wait_bounded(r.full + 8 * stage, phase, GEMV_WAIT_LIMIT_NS) || s_abort)
            {
                ok = false;
                s_abort = 1;
                break;
            }
            if (wait_cycles)
                *wait_cycles += (unsigned long long)(clock64() - c0);
            if (p.trace && tid == 0)
                trace_chunk(p.trace, cta, q, 0);
            if (wv < tiles)
            {
                const uint32_t st = r.ring + stage * GT_STAGE_BYTES;
                const bool two = wv + NC < tiles;
                const int ia = wv, ib = two ? wv + NC : wv;
                uint4 w0[2], w1[2];
                uint16_t sh0[2], sh1[2];
                uint32_t fa[2];
                float bsc[2];
#pragma unroll
                for (int k = 0; k < 2; ++k)
                {
                    const int i = k ? ib : ia, tt = c * CT + i;
                    w0[k] = lds128(st + i * 1024 + lane * 16);
                    w1[k] = lds128(st + i * 1024 + 512 + lane * 16);
                    const uint32_t sa = st + tiles * 1024 + i * 128 + lane * 2; // u16 scales
                    asm volatile("ld.shared.u16 %0, [%1];" : "=h"(sh0[k]) : "r"(sa));
                    asm volatile("ld.shared.u16 %0, [%1];" : "=h"(sh1[k]) : "r"(sa + 64));
                    fa[k] = f_base + (uint32_t)tt * f_step;
                    bsc[k] = ldsf(bs_base + (uint32_t)tt * 16);
                }
                int dp[2][4] = {}, dq[2][4] = {};
#pragma unroll
                for (int s = 0; s < 4; ++s)
                {
#pragma unroll
                    for (int k = 0; k < 2; ++k)
                    {
                        const uint32_t wa = u4get(w0[k], s), wb = u4get(w1[k], s);
                        const uint32_t a0 = wa & 0x0F0F0F0Fu, a1 = wb & 0x0F0F0F0Fu;
                        const uint32_t a2 = wa & 0xF0F0F0F0u, a3 = wb & 0xF0F0F0F0u;
                        const uint4 b = lds128(fa[k] + (uint32_t)s * f_sstep);
                        mma_u8s8_16832(dp[k][0], dp[k][1], dp[k][2], dp[k][3], a0, a1, a2, a3, b.x, b.y);
                        mma_u8s8_16832(dq[k][0], dq[k][1], dq[k][2], dq[k][3], a0, a1, a2, a3, b.z, b.w);
                    }
                }
#pragma unroll
                for (int k = 0; k < 2; ++k)
                {
                    if (k == 1 && !two)
                        break;
                    const float r0 = fmaf((float)(dq[k][0] * 128 + dq[k][1]), 1.0f / 16384.0f,
                                          (float)(dp[k][0] * 128 + dp[k][1]));
                    const float r1 = fmaf((float)(dq[k][2] * 128 + dq[k][3]), 1.0f / 16384.0f,
                                          (float)(dp[k][2] * 128 + dp[k][3]));
                    acc0 = fmaf(decode_scale<AAEDN_SCALE_F16>(sh0[k]) * bsc[k], r0, acc0);
                    acc1 = fmaf(decode_scale<AAEDN_SCALE_F16>(sh1[k]) * bsc[k], r1, acc1);
                }
            }
            __syncwarp();
            if (lane == 0)
                mbar_arrive(r.empty + 8 * stage);
            if (p.trace && tid == 0)
                trace_chunk(p.trace, cta, q, 1);
        }
        if (!ok)
            break;
        const int b = gl & (GT_RB - 1);
        float* rb = red + (size_t)b * NC * 16;
        unsigned* cnt = reinterpret_cast<unsigned*>(red + (size_t)GT_RB * NC * 16);
        acc0 += __shfl_xor_sync(0xffffffffu, acc0, 1);
        acc0 += __shfl_xor_sync(0xffffffffu, acc0, 2);
        acc1 += __shfl_xor_sync(0xffffffffu, acc1, 1);
        acc1 += __shfl_xor_sync(0xffffffffu, acc1, 2);
        if (t == 0)
        {
            rb[warp * 16 + g] = acc0;
            rb[warp * 16 + g + 8] = acc1;
        }
        __syncwarp();
        unsigned last = 0;
        if (lane == 0)
        {
            __threadfence_block();
            last = atomicAdd(cnt + b, 1u) == (unsigned)NC - 1 ? 1u : 0u;
        }
        last = __shfl_sync(0xffffffffu, last, 0);
        if (last)
        {
            __threadfence_block();
            float post = 1.0f;
            if constexpr (NORM)
            {
                float tss = 0.0f;
                for (int i = 0; i < NC; ++i) // fixed order
                    tss += wss[i];
                post = 1.0f / sqrtf(__fadd_rn(__fdiv_rn(tss, (float)p.K), p.eps)); // src/rmsnorm.cpp:34
            }
            gemv_epilogue<1, EPI, NC>(p, rb, group, lane, post, ecp, gl);
            __syncwarp();
            if (lane == 0)
                cnt[b] = 0u;
        }
    }
    return !named_bar_or(1, NCT, !ok);
}

// The decode GEMV kernel: one producer warp streaming the CTA's chunks, 16
// consumer warps with warp-built integer operands.
template <int PRO, int EPI>
__global__ void __launch_bounds__(GT_THREADS, 1) gemv_tiled_i8_kernel(const GemvParams p)
{
    const int NS = p.stages > 0 ? p.stages : GT_STAGES;
    constexpr int NC = GT_CONSUMERS;
    extern __shared__ __align__(16) uint8_t smem[];
    const int ntile = p.K >> 7;
    uint8_t* ring = smem;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + (size_t)NS * GT_STAGE_BYTES); // full[NS], empty[NS]
    uint4* frag = reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(bars) + (size_t)NS * 16);
    float* bscale = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(frag) + (size_t)ntile * 512);
    float* red = bscale + (size_t)ntile * 4;
    float* misc = red + GT_RED_BYTES / 4; // [32, 48) per-warp sums of squares, [48, 52) zero
    float* ecache = misc + 64;
    __shared__ int s_abort_mem;
    volatile int& s_abort = s_abort_mem;

    pdl_launch_dependents();
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (tid == 0)
        trace_mark(p.trace, blockIdx.x, 0);
    TiledRing r;
    r.ring = smem_addr(ring);
    r.full = smem_addr(bars);
    r.empty = r.full + NS * 8;
    r.ns = (uint32_t)NS;

    if (tid == 0)
    {
        for (int i = 0; i < NS; ++i)
        {
            mbar_init(r.full + 8 * i, 1);
            mbar_init(r.empty + 8 * i, NC);
        }
        mbar_init_fence();
        s_abort = 0;
    }
    if (tid < GT_RB)
        reinterpret_cast<unsigned*>(red + (size_t)GT_RB * NC * 16)[tid] = 0u;
    if (tid < 4)
        misc[48 + tid] = 0.0f;
    if (tid == 0)
        reinterpret_cast<unsigned*>(misc)[60] = 0u; // tensor parallel: the epoch warp 0 has seen
    __syncthreads();

    if (warp == NC)
    {
        // producer warp: the weights do not depend on the previous kernel
        uint32_t q = 0;
        if (!tiled_produce(p.w, p.N, p.K, r, q, blockIdx.x, gridDim.x, lane, nullptr, p.l2_hint != 0))
        {
            s_abort = 1;
            if (lane == 0 && p.state)
                p.state->err = 2u;
        }
        tiled_drain(r, q);
        return;
    }

    pdl_wait();
    if (tid == 0)
        trace_mark(p.trace, blockIdx.x, 2);
    warp_build_i8<PRO>(p, frag, bscale, misc + 32, nullptr, reinterpret_cast<volatile unsigned*>(misc + 60));
    if (tid == 0)
        trace_mark(p.trace, blockIdx.x, 1);
    uint32_t q = 0;
    if (!tiled_wb_consume<PRO, EPI>(p, r, q, frag, bscale, misc + 32, smem_addr(misc + 48), red, ecache,
                                    blockIdx.x, gridDim.x, s_abort))
    {
        if (lane == 0 && p.state)
            p.state->err = 2u;
    }
    else if (p.tp_sig)
    {
        // tensor parallel: the last CTA to finish copies this rank's partial
        // (complete: every CTA counted itself after a fence) into every other
        // rank's receive buffer, then raises this GEMV's epoch there
        volatile unsigned* last = reinterpret_cast<volatile unsigned*>(misc) + 61;
        __threadfence(); // every thread: its rows before the CTA counts itself
        named_bar_sync(1, NC * 32);
        if (tid == 0)
        {
            const bool l = atomicAdd(p.tp_counter, 1u) == gridDim.x - 1;
            if (l)
            {
                *p.tp_counter = 0u;
                __threadfence(); // the other CTAs' rows before the copy reads them
            }
            *last = l ? 1u : 0u;
        }
        named_bar_sync(1, NC * 32);
        if (*last)
        {
            const size_t off = ((size_t)p.tpc.rank * 2 + p.tp_buf) * p.tpc.dim;
            const float4* src = reinterpret_cast<const float4*>(p.tpc.recv[p.tpc.rank] + off);
            const int n4 = p.tpc.dim >> 2;
            for (int q = 0; q < p.tpc.size; ++q)
                if (q != p.tpc.rank)
                {
                    float4* dst = reinterpret_cast<float4*>(p.tpc.recv[q] + off);
                    for (int i = tid; i < n4; i += NC * 32)
                        dst[i] = __ldcg(src + i);
                }
            named_bar_sync(1, NC * 32);
            if (tid == 0)
                tp_signal(p.tpc, *p.tp_epoch + (unsigned)p.tp_sig_phase + 1u); // fences at system scope first
        }
    }
    if (tid == 0)
        trace_mark(p.trace, blockIdx.x, 3);
}

} // namespace aaedn_dev
