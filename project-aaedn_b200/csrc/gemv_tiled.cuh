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

#include "gemv_tma.cuh"

namespace aaedn_dev
{

constexpr int GT_CONSUMERS = 16;
constexpr int GT_THREADS = (GT_CONSUMERS + 1) * 32;
constexpr int GT_STAGES = 4;
constexpr int GT_CHUNK_TILES = 32; // two tiles per consumer warp
constexpr int GT_TILE_BYTES = 1024 + 128; // codes + scales of one tile (16 rows x 128 codes)
constexpr int GT_STAGE_BYTES = GT_CHUNK_TILES * GT_TILE_BYTES; // 36 KB

// Bytes of a repacked matrix (same as the row-major codes + scales).
inline size_t tiled_bytes(size_t N, size_t K) { return N * K / 2 + N * K / 32 * 2; }

// Repacks row-major codes/scales ([N][K], K % 128 == 0, N % 16 == 0).
void repack_tiled(const uint8_t* codes, const uint16_t* scales, size_t N, size_t K, uint8_t* out);

inline size_t gemv_tiled_smem_bytes(int ntile)
{
    return (size_t)GT_STAGES * GT_STAGE_BYTES + (size_t)GT_STAGES * 16 + (size_t)(ntile + 1) * 512 +
           (size_t)ntile * 16 + (size_t)2 * GT_CONSUMERS * 16 * 4 + 64 * 4;
}

template <int PRO, int EPI>
__global__ void __launch_bounds__(GT_THREADS, 1) gemv_tiled_kernel(const GemvParams p)
{
    constexpr int NS = GT_STAGES;
    constexpr int NC = GT_CONSUMERS;
    constexpr int NCT = NC * 32;
    constexpr int CT = GT_CHUNK_TILES;
    extern __shared__ __align__(16) uint8_t smem[];
    const int ntile = p.K >> 7; // the whole K: tiled weights are only used unchunked
    const int nchunk = (ntile + CT - 1) / CT;
    uint8_t* ring = smem;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + (size_t)NS * GT_STAGE_BYTES); // full[NS], empty[NS]
    uint4* frag = reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(bars) + (size_t)NS * 16);
    float* tb = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(frag) + (size_t)(ntile + 1) * 512);
    float* red = tb + (size_t)ntile * 4; // [2][NC][16]
    float* misc = red + 2 * NC * 16;
    __shared__ int s_abort_mem;
    volatile int& s_abort = s_abort_mem;

    pdl_launch_dependents();
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int n_groups = p.N >> 4;
    const int my_groups = blockIdx.x < n_groups ? (n_groups - 1 - blockIdx.x) / gridDim.x + 1 : 0;
    const uint32_t ring_a = smem_addr(ring);
    const uint32_t full_a = smem_addr(bars), empty_a = full_a + NS * 8;
    const size_t group_bytes = (size_t)ntile * GT_TILE_BYTES;

    if (tid == 0)
    {
        for (int i = 0; i < NS; ++i)
        {
            mbar_init(full_a + 8 * i, 1);
            mbar_init(empty_a + 8 * i, NC);
        }
        mbar_init_fence();
        s_abort = 0;
    }
    __syncthreads();

    if (warp == NC)
    {
        // ---------------- producer warp: one bulk copy per chunk ----------------
        uint32_t q = 0;
        bool ok = true;
        for (int gl = 0; gl < my_groups && ok; ++gl)
        {
            const uint8_t* gsrc = p.w + (size_t)(blockIdx.x + gl * gridDim.x) * group_bytes;
            for (int c = 0; c < nchunk; ++c, ++q)
            {
                const int tiles = (c + 1) * CT <= ntile ? CT : ntile - c * CT;
                const uint32_t stage = q % NS, use = q / NS;
                if (use > 0 && !mbar_wait_bounded(empty_a + 8 * stage, (use - 1) & 1, GEMV_WAIT_LIMIT_NS))
                {
                    ok = false;
                    break;
                }
                if (lane == 0)
                {
                    const uint32_t bytes = (uint32_t)tiles * GT_TILE_BYTES;
                    mbar_arrive_expect_tx(full_a + 8 * stage, bytes);
                    bulk_g2s(ring_a + stage * GT_STAGE_BYTES, gsrc + (size_t)c * CT * GT_TILE_BYTES, bytes,
                             full_a + 8 * stage);
                }
                __syncwarp();
            }
        }
        if (!ok)
        {
            s_abort = 1;
            if (lane == 0 && p.state)
                p.state->err = 2u;
        }
        // drain: every issued chunk has landed before the CTA may exit
        for (uint32_t k = (q > NS ? q - NS : 0); k < q; ++k)
            mbar_wait_bounded(full_a + 8 * (k % NS), (k / NS) & 1, GEMV_WAIT_LIMIT_NS);
        return;
    }

    // ---------------- consumer warps ----------------
    pdl_wait();
    gemv_build_frags<1, PRO, NCT>(p, frag, tb, misc, ntile);
    if (tid < 32)
        frag[(size_t)ntile * 32 + tid] = make_uint4(0, 0, 0, 0);
    named_bar_sync(1, NCT);

    const int g = lane >> 2, t = lane & 3;
    const bool bact = (g >> 1) == t;
    const int la = 2 * t + (g & 1);
    const uint32_t f_base = bact ? smem_addr(frag) + (uint32_t)la * 16 : smem_addr(frag) + (uint32_t)ntile * 512;
    const uint32_t f_step = bact ? 512u : 0u;
    const uint32_t tb_base = smem_addr(tb) + (uint32_t)t * 4;
    bool ok = true;
    uint32_t q = 0;
    for (int gl = 0; gl < my_groups; ++gl)
    {
        const int group = blockIdx.x + gl * gridDim.x;
        float acc0 = 0.0f, acc1 = 0.0f;
        for (int c = 0; c < nchunk && ok; ++c, ++q)
        {
            const int tiles = (c + 1) * CT <= ntile ? CT : ntile - c * CT;
            const uint32_t stage = q % NS;
            if (!mbar_wait_bounded(full_a + 8 * stage, (q / NS) & 1, GEMV_WAIT_LIMIT_NS) || s_abort)
            {
                ok = false;
                s_abort = 1;
                break;
            }
            if (warp < tiles)
            {
                const uint32_t st = ring_a + stage * GT_STAGE_BYTES;
                const bool two = warp + NC < tiles;
                const int ia = warp, ib = two ? warp + NC : warp;
                uint4 w0[2], w1[2];
                uint16_t sh0[2], sh1[2];
                uint32_t fa[2];
                float tbv[2];
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
                    tbv[k] = ldsf(tb_base + (uint32_t)tt * 16);
                }
                float d[2][2][4] = {}; // [tile][even/odd k-step][accumulator]
#pragma unroll
                for (int qq = 0; qq < 4; ++qq)
                {
#pragma unroll
                    for (int k = 0; k < 2; ++k)
                    {
                        const uint32_t wa = u4get(w0[k], qq), wb = u4get(w1[k], qq);
                        const uint4 b = lds128(fa[k] + qq * 128);
                        float* dd = d[k][qq & 1];
                        mma_bf16_16816(dd[0], dd[1], dd[2], dd[3], nib_e0(wa), nib_e0(wb), nib_e1(wa), nib_e1(wb),
                                       b.x, b.y);
                        mma_bf16_16816(dd[0], dd[1], dd[2], dd[3], nib_e2(wa), nib_e2(wb), nib_e3(wa), nib_e3(wb),
                                       b.z, b.w);
                    }
                }
#pragma unroll
                for (int k = 0; k < 2; ++k)
                {
                    if (k == 1 && !two)
                        break;
                    const float sc0 = decode_scale<AAEDN_SCALE_F16>(sh0[k]);
                    const float sc1 = decode_scale<AAEDN_SCALE_F16>(sh1[k]);
                    acc0 = fmaf(sc0, ((d[k][0][0] + d[k][1][0]) + (d[k][0][1] + d[k][1][1])) - tbv[k], acc0);
                    acc1 = fmaf(sc1, ((d[k][0][2] + d[k][1][2]) + (d[k][0][3] + d[k][1][3])) - tbv[k], acc1);
                }
            }
            __syncwarp();
            if (lane == 0)
                mbar_arrive(empty_a + 8 * stage);
        }
        float* rb = red + (size_t)(gl & 1) * NC * 16;
        acc0 += __shfl_xor_sync(0xffffffffu, acc0, 1);
        acc0 += __shfl_xor_sync(0xffffffffu, acc0, 2);
        acc1 += __shfl_xor_sync(0xffffffffu, acc1, 1);
        acc1 += __shfl_xor_sync(0xffffffffu, acc1, 2);
        if (t == 0)
        {
            rb[warp * 16 + g] = acc0;
            rb[warp * 16 + g + 8] = acc1;
        }
        named_bar_sync(1, NCT);
        if (!ok || s_abort)
        {
            if (lane == 0 && p.state)
                p.state->err = 2u;
            break;
        }
        if (warp == (gl & (NC - 1)))
            gemv_epilogue<1, EPI, NC>(p, rb, group, lane);
    }
}

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

__device__ __forceinline__ uint32_t pack_s8x4(int a, int b, int c, int d)
{
    return (uint32_t)(a & 0xFF) | ((uint32_t)(b & 0xFF) << 8) | ((uint32_t)(c & 0xFF) << 16) |
           ((uint32_t)(d & 0xFF) << 24);
}

// Base-128 digits of v, |v| <= 127.5.
__device__ __forceinline__ void digits4(float v, int (&d)[4])
{
    float r = fminf(fmaxf(rintf(v), -127.0f), 127.0f);
    d[0] = (int)r;
    r = (v - r) * 128.0f; // exact: |v - rint(v)| <= 1/2 (plus the clamp)
#pragma unroll
    for (int i = 1; i < 4; ++i)
    {
        const float q = rintf(r);
        d[i] = (int)q;
        r = (r - q) * 128.0f;
    }
}

// Writes the B operands of tiles [0, ntile) to frag[tile][word s][lane g][4
// words] (16 B; the active lanes are g = 2*tb + j for block tb of the tile
// and digit parity j: words (digit j even-code elements, digit j odd, digit
// 2+j even, digit 2+j odd)) and the zero tile after them; misc[0] receives
// the output factor max|x| / (127 * 128). NTH threads (named barrier 1).
template <int PRO, int NTH>
__device__ __forceinline__ void gemv_build_i8(const GemvParams& p, uint4* frag, float* misc, int ntile)
{
    const int tid = threadIdx.x;
    const float* src = p.x;
    if constexpr (PRO == PRO_EMBED_RMSNORM)
    {
        const uint32_t pos = p.state->pos;
        const uint32_t tok = pos < p.state->n_prompt ? p.prompt[pos] : p.state->next_token;
        src = p.embedding + (size_t)tok * p.K;
        if (blockIdx.x == 0)
            for (int i = tid; i < p.K; i += NTH)
                p.hidden_out[i] = src[i];
    }
    // pass 1: sum of squares (RMSNorm) and the largest |v * gain|
    float ss = 0.0f, mx = 0.0f;
    bool finite = true;
    {
        const float4* s4 = reinterpret_cast<const float4*>(src);
        const float4* g4 = reinterpret_cast<const float4*>(p.gain);
        for (int i = tid; i < (p.K >> 2); i += NTH)
        {
            const float4 v = s4[i];
            float4 a = v;
            if constexpr (PRO != PRO_PLAIN)
            {
                ss = fmaf(v.x, v.x, ss);
                ss = fmaf(v.y, v.y, ss);
                ss = fmaf(v.z, v.z, ss);
                ss = fmaf(v.w, v.w, ss);
                const float4 g = g4[i];
                a = make_float4(v.x * g.x, v.y * g.y, v.z * g.z, v.w * g.w);
            }
            const float m4 = fmaxf(fmaxf(fabsf(a.x), fabsf(a.y)), fmaxf(fabsf(a.z), fabsf(a.w)));
            finite = finite && (m4 <= 3.0e38f) && (a.x == a.x) && (a.y == a.y) && (a.z == a.z) && (a.w == a.w);
            mx = fmaxf(mx, m4);
        }
    }
    float rms = 1.0f;
    if constexpr (PRO != PRO_PLAIN)
    {
        ss = group_sum<NTH>(ss, misc);
        rms = 1.0f / sqrtf(__fadd_rn(__fdiv_rn(ss, (float)p.K), p.eps)); // src/rmsnorm.cpp:34
    }
    // block-wide max; a non-finite activation makes every output NaN
    mx = finite ? mx : __int_as_float(0x7f800000);
    mx = warp_max(mx);
    named_bar_sync(1, NTH);
    if ((tid & 31) == 0)
        misc[8 + (tid >> 5)] = mx;
    named_bar_sync(1, NTH);
    mx = 0.0f;
    for (int i = 0; i < NTH / 32; ++i)
        mx = fmaxf(mx, misc[8 + i]);
    mx *= rms;
    const bool bad = !(mx <= 3.0e38f);
    const float inv = (mx > 0.0f && !bad) ? 127.0f / mx : 0.0f;
    // pass 2: the digits, 8 elements (one code word of one block) per item
    const int items = ntile * 16;
    for (int it = tid; it < items; it += NTH)
    {
        const int tile = it >> 4, tb = (it >> 2) & 3, s = it & 3;
        const int k0 = tile * 128 + tb * 32 + s * 8;
        const float4 a = *reinterpret_cast<const float4*>(src + k0);
        const float4 b = *reinterpret_cast<const float4*>(src + k0 + 4);
        float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
        if constexpr (PRO != PRO_PLAIN)
        {
            const float4 ga = *reinterpret_cast<const float4*>(p.gain + k0);
            const float4 gb = *reinterpret_cast<const float4*>(p.gain + k0 + 4);
            const float gv[8] = {ga.x, ga.y, ga.z, ga.w, gb.x, gb.y, gb.z, gb.w};
#pragma unroll
            for (int c = 0; c < 8; ++c)
                v[c] = __fmul_rn(__fmul_rn(v[c], rms), gv[c]); // src/rmsnorm.cpp:42-43
        }
        int d[8][4];
#pragma unroll
        for (int c = 0; c < 8; ++c)
        {
            // even elements as y, odd ones as y/16 (their codes enter as 16*c)
            const float y = __fmul_rn(v[c], inv) * ((c & 1) ? 0.0625f : 1.0f);
            digits4(y, d[c]);
        }
        uint4* dst = frag + ((size_t)tile * 4 + s) * 8 + 2 * tb;
#pragma unroll
        for (int j = 0; j < 2; ++j)
            dst[j] = make_uint4(pack_s8x4(d[0][j], d[2][j], d[4][j], d[6][j]),
                                pack_s8x4(d[1][j], d[3][j], d[5][j], d[7][j]),
                                pack_s8x4(d[0][2 + j], d[2][2 + j], d[4][2 + j], d[6][2 + j]),
                                pack_s8x4(d[1][2 + j], d[3][2 + j], d[5][2 + j], d[7][2 + j]));
    }
    if (tid < 32)
        frag[(size_t)ntile * 32 + tid] = make_uint4(0, 0, 0, 0);
    if (tid == 0)
        misc[0] = bad ? __int_as_float(0x7fc00000) : mx / (127.0f * 128.0f);
    named_bar_sync(1, NTH);
}

inline size_t gemv_tiled_i8_smem_bytes(int ntile)
{
    return (size_t)GT_STAGES * GT_STAGE_BYTES + (size_t)GT_STAGES * 16 + (size_t)(ntile + 1) * 512 +
           (size_t)2 * GT_CONSUMERS * 16 * 4 + 64 * 4;
}

// Same CTA shape, ring and layout as gemv_tiled_kernel; the consumers use the
// integer engine above.
template <int PRO, int EPI>
__global__ void __launch_bounds__(GT_THREADS, 1) gemv_tiled_i8_kernel(const GemvParams p)
{
    constexpr int NS = GT_STAGES;
    constexpr int NC = GT_CONSUMERS;
    constexpr int NCT = NC * 32;
    constexpr int CT = GT_CHUNK_TILES;
    extern __shared__ __align__(16) uint8_t smem[];
    const int ntile = p.K >> 7;
    const int nchunk = (ntile + CT - 1) / CT;
    uint8_t* ring = smem;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + (size_t)NS * GT_STAGE_BYTES); // full[NS], empty[NS]
    uint4* frag = reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(bars) + (size_t)NS * 16);
    float* red = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(frag) + (size_t)(ntile + 1) * 512);
    float* misc = red + 2 * NC * 16; // [0] output factor, [8..8+NC) max scratch
    __shared__ int s_abort_mem;
    volatile int& s_abort = s_abort_mem;

    pdl_launch_dependents();
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int n_groups = p.N >> 4;
    const int my_groups = blockIdx.x < n_groups ? (n_groups - 1 - blockIdx.x) / gridDim.x + 1 : 0;
    const uint32_t ring_a = smem_addr(ring);
    const uint32_t full_a = smem_addr(bars), empty_a = full_a + NS * 8;
    const size_t group_bytes = (size_t)ntile * GT_TILE_BYTES;

    if (tid == 0)
    {
        for (int i = 0; i < NS; ++i)
        {
            mbar_init(full_a + 8 * i, 1);
            mbar_init(empty_a + 8 * i, NC);
        }
        mbar_init_fence();
        s_abort = 0;
    }
    __syncthreads();

    if (warp == NC)
    {
        // ---------------- producer warp: one bulk copy per chunk ----------------
        uint32_t q = 0;
        bool ok = true;
        for (int gl = 0; gl < my_groups && ok; ++gl)
        {
            const uint8_t* gsrc = p.w + (size_t)(blockIdx.x + gl * gridDim.x) * group_bytes;
            for (int c = 0; c < nchunk; ++c, ++q)
            {
                const int tiles = (c + 1) * CT <= ntile ? CT : ntile - c * CT;
                const uint32_t stage = q % NS, use = q / NS;
                if (use > 0 && !mbar_wait_bounded(empty_a + 8 * stage, (use - 1) & 1, GEMV_WAIT_LIMIT_NS))
                {
                    ok = false;
                    break;
                }
                if (lane == 0)
                {
                    const uint32_t bytes = (uint32_t)tiles * GT_TILE_BYTES;
                    mbar_arrive_expect_tx(full_a + 8 * stage, bytes);
                    bulk_g2s(ring_a + stage * GT_STAGE_BYTES, gsrc + (size_t)c * CT * GT_TILE_BYTES, bytes,
                             full_a + 8 * stage);
                }
                __syncwarp();
            }
        }
        if (!ok)
        {
            s_abort = 1;
            if (lane == 0 && p.state)
                p.state->err = 2u;
        }
        // drain: every issued chunk has landed before the CTA may exit
        for (uint32_t k = (q > NS ? q - NS : 0); k < q; ++k)
            mbar_wait_bounded(full_a + 8 * (k % NS), (k / NS) & 1, GEMV_WAIT_LIMIT_NS);
        return;
    }

    // ---------------- consumer warps ----------------
    pdl_wait();
    gemv_build_i8<PRO, NCT>(p, frag, misc, ntile);
    const float out_scale = misc[0];

    const int g = lane >> 2, t = lane & 3;
    const bool bact = (g >> 1) == t;
    // active lanes read their own 16 B of every (tile, word) row of the
    // fragments; the others read the zero tile
    const uint32_t f_base = bact ? smem_addr(frag) + (uint32_t)g * 16 : smem_addr(frag) + (uint32_t)ntile * 512;
    const uint32_t f_step = bact ? 512u : 0u;
    const uint32_t f_sstep = bact ? 128u : 0u;
    bool ok = true;
    uint32_t q = 0;
    for (int gl = 0; gl < my_groups; ++gl)
    {
        const int group = blockIdx.x + gl * gridDim.x;
        float acc0 = 0.0f, acc1 = 0.0f;
        for (int c = 0; c < nchunk && ok; ++c, ++q)
        {
            const int tiles = (c + 1) * CT <= ntile ? CT : ntile - c * CT;
            const uint32_t stage = q % NS;
            if (!mbar_wait_bounded(full_a + 8 * stage, (q / NS) & 1, GEMV_WAIT_LIMIT_NS) || s_abort)
            {
                ok = false;
                s_abort = 1;
                break;
            }
            if (warp < tiles)
            {
                const uint32_t st = ring_a + stage * GT_STAGE_BYTES;
                const bool two = warp + NC < tiles;
                const int ia = warp, ib = two ? warp + NC : warp;
                uint4 w0[2], w1[2];
                uint16_t sh0[2], sh1[2];
                uint32_t fa[2];
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
                }
                int dp[2][4] = {}, dq[2][4] = {}; // [tile][accumulator]: digits (0,1) and (2,3)
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
                    // lane (g, t) holds block t of the tile for rows g and g + 8:
                    // digits (0,1) in dp, (2,3) in dq; |dp[0]*128 + dp[1]| < 2^24
                    const float r0 = fmaf((float)(dq[k][0] * 128 + dq[k][1]), 1.0f / 16384.0f,
                                          (float)(dp[k][0] * 128 + dp[k][1]));
                    const float r1 = fmaf((float)(dq[k][2] * 128 + dq[k][3]), 1.0f / 16384.0f,
                                          (float)(dp[k][2] * 128 + dp[k][3]));
                    acc0 = fmaf(decode_scale<AAEDN_SCALE_F16>(sh0[k]), r0, acc0);
                    acc1 = fmaf(decode_scale<AAEDN_SCALE_F16>(sh1[k]), r1, acc1);
                }
            }
            __syncwarp();
            if (lane == 0)
                mbar_arrive(empty_a + 8 * stage);
        }
        float* rb = red + (size_t)(gl & 1) * NC * 16;
        acc0 += __shfl_xor_sync(0xffffffffu, acc0, 1);
        acc0 += __shfl_xor_sync(0xffffffffu, acc0, 2);
        acc1 += __shfl_xor_sync(0xffffffffu, acc1, 1);
        acc1 += __shfl_xor_sync(0xffffffffu, acc1, 2);
        if (t == 0)
        {
            rb[warp * 16 + g] = acc0 * out_scale;
            rb[warp * 16 + g + 8] = acc1 * out_scale;
        }
        named_bar_sync(1, NCT);
        if (!ok || s_abort)
        {
            if (lane == 0 && p.state)
                p.state->err = 2u;
            break;
        }
        if (warp == (gl & (NC - 1)))
            gemv_epilogue<1, EPI, NC>(p, rb, group, lane);
    }
}

} // namespace aaedn_dev
