// gemv_tiled.cuh — the decode dequant-GEMV over tile-major ("tiled") weights.
//
// The model repacks every quantized matrix once at load time. The blocks and
// scales are the reference's (32 codes = 16 bytes, one fp16 scale per block);
// only their order in memory changes, so that everything one step of the
// consumers needs is one contiguous run:
//   matrix = row groups of 16 rows, in order
//   group  = chunks of up to 16 tiles (a tile = 128 codes = 4 quant blocks of
//            each of the 16 rows = 1 KB of codes); the last chunk of a group
//            may be short
//   chunk  = the tiles' codes, then the tiles' scales
//   tile codes  = [pair P][lane l][16 B]: lane l = 4g + t holds, for rows g
//                 and g + 8 (r = 0, 1) and halves H = 0, 1, the 4 bytes
//                 [8H + 4(t & 1), +4) of block 2P + (t >> 1): words (H0 r0,
//                 H0 r1, H1 r0, H1 r1) = the A fragments of the two mmas of
//                 pair P;
//   tile scales = [P][g][b'][r] u16: block 2P + b' of row g + 8r.
// A row group's K range is one linear stream, so one bulk (TMA) copy moves a
// whole chunk (up to 18 KB) and DRAM sees long sequential bursts; a warp's
// 16-byte reads of a tile cover 512 consecutive shared-memory bytes (no bank
// conflicts).
//
// CTA: one producer warp (bulk copies into a ring of up to 12 stages,
// mbarriers) + 24 consumer warps in 6 groups of 4; chunk q of the CTA's
// stream goes to group q % 6, whose warp j takes tiles 4j..4j+3 of it, so
// six chunks are worked on at once and a warp's four tiles give it 16
// independent mmas per chunk.
#pragma once

#include "gemv_q4.cuh"

namespace aaedn_dev
{

constexpr uint64_t GEMV_WAIT_LIMIT_NS = 2000000000ull; // 2 s: bound of every mbarrier wait

constexpr int GT_CONSUMERS = 24;
constexpr int GT_GROUPS = 6;                             // consumer groups (chunks in flight at once)
constexpr int GT_GROUP_WARPS = GT_CONSUMERS / GT_GROUPS; // warps of a group
constexpr int GT_THREADS = (GT_CONSUMERS + 1) * 32;
// Ring stages (any number: the producer tags each stage with the chunk it
// holds, and a consumer waits for its chunk's tag before the parity wait).
constexpr int GT_STAGES = 2;     // fewest ring stages a launch takes
constexpr int GT_MAX_STAGES = 12;
constexpr int GT_CHUNK_TILES = 16; // four tiles per warp of a group
constexpr int GT_TILE_BYTES = 1024 + 128; // codes + scales of one tile (16 rows x 128 codes)
constexpr int GT_STAGE_BYTES = GT_CHUNK_TILES * GT_TILE_BYTES; // 18 KB
constexpr int GT_FRAG_TILE_BYTES = 512; // activation digits of one tile (B fragments)
// A block's activation is scaled to |y| <= 119 before its digits are taken:
// the top digit of odd - even (up to 119 * 17 / 16) then fits a signed byte.
constexpr float GT_YMAX = 119.0f;
// Partial sums in flight: slot q % GT_RQ holds chunk q's [4 warps][16 rows];
// row group counters by group number % GT_RC. Chunks in flight are bounded by
// the ring (stages + the groups' current chunks), row groups by those over
// the chunks per group: 32 covers 12 stages and 16 chunks per row group.
constexpr int GT_RQ = 32;
constexpr int GT_RC = 32;
constexpr int GT_RED_BYTES = GT_RQ * GT_GROUP_WARPS * 16 * 4 + GT_RC * 4 + GT_CONSUMERS * 16 * 4;
// The CTA's small shared words (floats): per-warp sums of squares at WSS,
// 16 zero bytes at ZERO, flags, and the ring's stage tags at TAG.
constexpr int GT_MISC_WSS = 0, GT_MISC_ZERO = 32, GT_MISC_FLAG = 40, GT_MISC_LAST = 41, GT_MISC_TAG = 48;
constexpr int GT_MISC_FLOATS = 64;
static_assert(GT_CONSUMERS <= GT_MISC_ZERO, "per-warp sums overlap the zero words");
constexpr int GT_MAX_CHUNKS = 16; // chunks per row group: K <= 32768
// Shared memory for the staged epilogue inputs (EpiCache): 2048 floats.
constexpr int GT_ECACHE_FLOATS = 2048;

// Bytes of a repacked matrix (same as the row-major codes + scales).
inline size_t tiled_bytes(size_t N, size_t K) { return N * K / 2 + N * K / 32 * 2; }

// Repacks row-major codes/scales ([N][K], K % 128 == 0, N % 16 == 0).
void repack_tiled(const uint8_t* codes, const uint16_t* scales, size_t N, size_t K, uint8_t* out);

// ---------------------------------------------------------------------------
// Integer dot-product engine.
//
// The activation x (after the prologue) is scaled per 32-element block to
// y = x * 127 / max|x| and written as four signed base-128 digits of
// Y = round(y * 2^21) = d0 2^21 + d1 2^14 + d2 2^7 + d3 (d0 in [-127, 127],
// the others in [-64, 64]; odd elements carry y / 16, see below), so that a
// block's dot product with the 4-bit codes is four exact integer sums,
// computed by the u8 x s8 mma (m16n8k32). The codes stay as they are in
// memory: the low nibble of every byte (even element) is fed as c, the high
// nibble in place as 16 c, and the odd elements' digits are those of y / 16
// to match. One mma covers 16 codes of each of two blocks (lanes t = 0, 1 of
// a quad hold block 2P, lanes 2, 3 block 2P + 1); its 8 columns are (block,
// digit) pairs, so it yields all four digit sums of both blocks, and the two
// halves H of a block add into the same accumulators: four mmas per tile,
// nothing rounded inside the integer products. Lane t of a quad ends with
// digits (2(t & 1), 2(t & 1) + 1) of block 2P + (t >> 1) for rows g, g + 8;
// the quad's sum over t is the tile's dot product.
// ---------------------------------------------------------------------------

inline size_t gemv_tiled_i8_smem_bytes(int ntile, int stages = GT_STAGES)
{
    return (size_t)stages * GT_STAGE_BYTES + (size_t)stages * 16 + (size_t)ntile * (GT_FRAG_TILE_BYTES + 32) +
           GT_RED_BYTES + GT_MISC_FLOATS * 4 + GT_ECACHE_FLOATS * 4;
}

// The most ring stages (<= GT_MAX_STAGES) whose shared memory fits `budget`.
inline int gemv_tiled_stages(int ntile, size_t budget)
{
    int s = GT_MAX_STAGES;
    while (s > GT_STAGES && gemv_tiled_i8_smem_bytes(ntile, s) > budget)
        --s;
    return s;
}

// The shared-memory ring of a tiled GEMV CTA: stage i at ring + i * 18 KB,
// full[i] / empty[i] mbarriers, tag[i] = the chunk it was last issued for.
// Chunks are numbered in the order the producer issues them (q); chunk q
// sits in stage q % ns, use q / ns.
struct TiledRing
{
    uint32_t ring, full, empty, tag; // shared-memory addresses
    uint32_t ns;                     // stages
};

__device__ __forceinline__ void st_shared_u32_volatile(uint32_t addr, uint32_t v)
{
    asm volatile("st.volatile.shared.u32 [%0], %1;" ::"r"(addr), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_shared_u32_volatile(uint32_t addr)
{
    uint32_t v;
    asm volatile("ld.volatile.shared.u32 %0, [%1];" : "=r"(v) : "r"(addr) : "memory");
    return v;
}

// A consumer's wait for chunk qq (stage st, use `use`). The stage's previous
// use may belong to another group and may not have landed when this group
// arrives, so a parity bit alone could match that pending phase. Once the
// stage is tagged qq, the producer has seen the previous use consumed (it
// waits for that before tagging), so the stage has completed `use` or
// `use + 1` fills, which the parity of `use` tells apart.
__device__ __forceinline__ bool tiled_wait_chunk(const TiledRing& r, uint32_t qq, uint32_t st, uint32_t use)
{
    const uint32_t tag = r.tag + 4 * st;
    if (ld_shared_u32_volatile(tag) != qq)
    {
        const uint64_t t0 = globaltimer_ns();
        while (ld_shared_u32_volatile(tag) != qq)
            if (globaltimer_ns() - t0 > GEMV_WAIT_LIMIT_NS)
                return false;
    }
    return mbar_wait_bounded(r.full + 8 * st, use & 1, GEMV_WAIT_LIMIT_NS);
}

// Producer warp: issues, for every row group this CTA owns (cta, cta + ncta,
// ...), its chunks of the tile-major matrix w ([N/16][K/128 tiles]). Returns
// false if a wait for a free stage ran out (the caller drains and stops).
__device__ __forceinline__ bool tiled_produce(const uint8_t* w, int N, int K, const TiledRing& r, uint32_t& q,
                                              int cta, int ncta, int lane, bool hint = false)
{
    constexpr int CT = GT_CHUNK_TILES;
    const uint32_t NS = r.ns;
    const int ntile = K >> 7, nchunk = (ntile + CT - 1) / CT, n_groups = N >> 4;
    const size_t group_bytes = (size_t)ntile * GT_TILE_BYTES;
    uint32_t stage = q % NS, use = q / NS; // advanced without a division per chunk
    for (int group = cta; group < n_groups; group += ncta)
    {
        const uint8_t* gsrc = w + (size_t)group * group_bytes;
        for (int c = 0; c < nchunk; ++c, ++q, (++stage == NS) ? (stage = 0, ++use) : 0u)
        {
            const int tiles = (c + 1) * CT <= ntile ? CT : ntile - c * CT;
            if (use > 0 && !mbar_wait_bounded(r.empty + 8 * stage, (use - 1) & 1, GEMV_WAIT_LIMIT_NS))
                return false;
            if (lane == 0)
            {
                st_shared_u32_volatile(r.tag + 4 * stage, q); // the previous use is consumed
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
// The activation operand, built by the 24 consumer warps together.
//
// Work item = 8 elements (codes 8s..8s+7 of block tb of a tile); the 4 items
// of a block sit in one lane quad, which finds the block's max with two
// shuffles. Fragment layout: frag[tile][P][slot][16 B], slot = 2 g + h for
// the mma column g = 4 b' + d (block 2P + b', digit d) and the half h of the
// block's byte pairs (t & 1 of the consuming lane); the 16 bytes are (H = 0:
// b0, b1; H = 1: b0, b1), b0 holding digit d of the 4 even elements of those
// bytes (met by the raw code bytes), b1 digit d of odd - even (met by the
// high nibbles). bscale[(tile * 4 + t) * 2 + P] = the unit max / (119 * 128)
// of block 2P + (t >> 1), times 2^-14 for t odd (the lanes holding digits
// 2 and 3). The RMSNorm factor stays out: a scalar applied after the dot
// product, from the per-warp sums of squares in wss.
// ---------------------------------------------------------------------------
template <int PRO>
__device__ __forceinline__ void gt_build(const GemvParams& p, uint8_t* frag, float* bscale, float* wss)
{
    constexpr bool NORM = PRO == PRO_RMSNORM || PRO == PRO_EMBED_RMSNORM;
    constexpr int NCT = GT_CONSUMERS * 32;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int ntile = p.K >> 7, nitems = ntile * 16;
    const float* src = p.x;
    if constexpr (PRO == PRO_EMBED_RMSNORM)
    {
        const uint32_t pos = p.state->pos;
        const uint32_t tok = pos < p.state->n_prompt ? p.prompt[pos] : p.state->next_token;
        src = p.embedding + (size_t)tok * p.lda;
    }
    float ss = 0.0f;
    // items in batches of MAXI per thread, each batch's loads first (one L2
    // round trip per batch: one batch up to K = 16384)
    constexpr int MAXI = 4;
    for (int ib = 0; ib * MAXI * NCT < nitems; ++ib)
    {
    float v[MAXI][8];
#pragma unroll
    for (int it = 0; it < MAXI; ++it)
    {
        const int item = tid + (ib * MAXI + it) * NCT;
        const int k0 = item * 8;
#pragma unroll
        for (int c = 0; c < 8; ++c)
            v[it][c] = 0.0f;
        if (item < nitems)
        {
            const float4 a = __ldcg(reinterpret_cast<const float4*>(src + k0));
            const float4 b = __ldcg(reinterpret_cast<const float4*>(src + k0 + 4));
            v[it][0] = a.x, v[it][1] = a.y, v[it][2] = a.z, v[it][3] = a.w;
            v[it][4] = b.x, v[it][5] = b.y, v[it][6] = b.z, v[it][7] = b.w;
            if constexpr (PRO == PRO_EMBED_RMSNORM)
                if (blockIdx.x == 0)
                {
                    *reinterpret_cast<float4*>(p.hidden_out + k0) = a;
                    *reinterpret_cast<float4*>(p.hidden_out + k0 + 4) = b;
                }
            if constexpr (NORM)
            {
                const float4 ga = __ldg(reinterpret_cast<const float4*>(p.gain + k0));
                const float4 gb = __ldg(reinterpret_cast<const float4*>(p.gain + k0 + 4));
                const float gv[8] = {ga.x, ga.y, ga.z, ga.w, gb.x, gb.y, gb.z, gb.w};
#pragma unroll
                for (int c = 0; c < 8; ++c)
                {
                    ss = fmaf(v[it][c], v[it][c], ss);
                    v[it][c] = __fmul_rn(v[it][c], gv[c]); // src/rmsnorm.cpp:42-43 without the 1/rms
                }
            }
        }
    }
#pragma unroll
    for (int it = 0; it < MAXI; ++it)
    {
        const int item = tid + (ib * MAXI + it) * NCT;
        if ((ib * MAXI + it) * NCT >= nitems)
            break; // uniform over the CTA
        const int tile = item >> 4, tb = (item >> 2) & 3, s = item & 3;
        // block max over the quad (the block's 4 items); a non-finite value
        // makes the block's unit NaN (so its outputs are)
        float mx = 0.0f;
        bool fin = true;
#pragma unroll
        for (int c = 0; c < 8; ++c)
        {
            const float a8 = fabsf(v[it][c]);
            fin = fin && (a8 <= 3.0e38f);
            mx = fmaxf(mx, a8);
        }
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
        const unsigned bad = __ballot_sync(0xffffffffu, !fin);
        const bool bbad = ((bad >> (lane & ~3)) & 0xFu) != 0;
        const float inv = (mx > 0.0f && !bbad) ? GT_YMAX / mx : 0.0f;
        if (item < nitems)
        {
            // Y = round(y * 2^21) for an even element, round(y * 2^17) (of
            // y/16) for an odd one; the mma's raw-byte half meets the even
            // element's Y, its high-nibble half the difference odd - even:
            // (lo + 16 hi) Ye + 16 hi (Yo - Ye) = lo Ye + 16 hi Yo. Both as
            // balanced base-128 digits, exact integer arithmetic.
            int Yv[8];
#pragma unroll
            for (int cc = 0; cc < 8; ++cc)
                Yv[cc] = __float2int_rn(__fmul_rn(v[it][cc], inv) * ((cc & 1) ? 131072.0f : 2097152.0f));
            int dg[8][4];
#pragma unroll
            for (int cc = 0; cc < 8; ++cc)
            {
                const int Y = (cc & 1) ? Yv[cc] - Yv[cc - 1] : Yv[cc];
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
            // these 8 elements are bytes 4s..4s+3 of block tb: pair P = tb / 2,
            // b' = tb % 2, half H = s / 2, slot half h = s % 2
            const int P = tb >> 1, bp = tb & 1, H = s >> 1, h = s & 1;
            uint8_t* base = frag + ((size_t)tile * 2 + P) * 256 + H * 8;
#pragma unroll
            for (int d = 0; d < 4; ++d)
                *reinterpret_cast<uint2*>(base + (2 * (4 * bp + d) + h) * 16) = make_uint2(pack(0, d), pack(1, d));
            // the block's unit, for the consuming lanes t = 2 b' + h (h = 1:
            // digits (2, 3), weight 2^-14), component P of their pair
            if (s < 2)
            {
                const float u = mx / (GT_YMAX * 128.0f);
                bscale[(tile * 4 + 2 * bp + s) * 2 + P] =
                    bbad ? __int_as_float(0x7fc00000) : (s ? __fmul_rn(u, 1.0f / 16384.0f) : u);
            }
        }
    }
    }
    if constexpr (NORM)
    {
        ss = warp_sum(ss);
        if (lane == 0)
            wss[warp] = ss;
    }
}

// Consumer warps of one GEMV (after gt_build and a consumer barrier).
template <int PRO, int EPI>
__device__ __forceinline__ bool gt_consume(const GemvParams& p, const TiledRing& r, uint32_t q0, const uint8_t* frag,
                                           const float* bscale, const float* wss, uint32_t zero16, float* red,
                                           float* ecache, int cta, int ncta, volatile int& s_abort)
{
    constexpr bool NORM = PRO == PRO_RMSNORM || PRO == PRO_EMBED_RMSNORM;
    constexpr int NCT = GT_CONSUMERS * 32;
    constexpr int CT = GT_CHUNK_TILES;
    const uint32_t NS = r.ns;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int grp = warp >> 2, wj = warp & 3; // group, warp of the group
    const int ntile = p.K >> 7, nchunk = (ntile + CT - 1) / CT, n_groups = p.N >> 4;
    const int my_groups = cta < n_groups ? (n_groups - 1 - cta) / ncta + 1 : 0;
    const int g = lane >> 2, t = lane & 3;
    const bool bact = (t >> 1) == (g >> 2);
    const uint32_t f_base = bact ? smem_addr(frag) + (uint32_t)(2 * g + (t & 1)) * 16 : zero16;
    const uint32_t f_tile = bact ? (uint32_t)GT_FRAG_TILE_BYTES : 0u, f_pair = bact ? 256u : 0u;
    const uint32_t bs_base = smem_addr(bscale) + (uint32_t)t * 8; // (pair 0, pair 1) units of this lane's class
    float* part = red;                                                     // [RQ][4][16]
    unsigned* cnt = reinterpret_cast<unsigned*>(red + GT_RQ * GT_GROUP_WARPS * 16); // [RC]
    float* tmp = reinterpret_cast<float*>(cnt + GT_RC) + warp * 16;          // this warp's 16 sums
    // epilogue inputs into shared memory (read by whichever warp completes a
    // row group; staged before the consumer barrier that follows the build)
    EpiCache ec{};
    const EpiCache* ecp = nullptr;
    if constexpr (EPI == EPI_RESIDUAL)
    {
        if (my_groups * 16 <= GT_ECACHE_FLOATS)
        {
            ec.resid = ecache;
            ecp = &ec;
        }
    }
    else if constexpr (EPI == EPI_QKV_ROPE)
    {
        const uint32_t pos = p.state->pos;
        if ((p.head_dim >> 1) <= GT_ECACHE_FLOATS / 2 && pos < (uint32_t)p.max_pos)
        {
            ec.cos = ecache;
            ec.sin = ecache + GT_ECACHE_FLOATS / 2;
            ec.page = __ldg(p.page_table + pos / p.page_size);
            ecp = &ec;
        }
    }
    const int nq = my_groups * nchunk;
    bool ok = true;
    // chunk q = grp, grp + GT_GROUPS, ...: its stage, use, row group and chunk
    // within the row group are advanced without divisions
    uint32_t qq = q0 + (uint32_t)grp, stage = qq % NS, use = qq / NS;
    int gl = grp / nchunk, c = grp - gl * nchunk;
    for (int q = grp; q < nq; q += GT_GROUPS)
    {
        const int tiles = (c + 1) * CT <= ntile ? CT : ntile - c * CT;
        if (!tiled_wait_chunk(r, qq, stage, use) || s_abort)
        {
            ok = false;
            s_abort = 1;
            break;
        }
        if (p.trace && tid == 0)
            trace_chunk(p.trace, cta, qq, 0);
        float2 acc = make_float2(0.0f, 0.0f); // rows g, g + 8
        const uint32_t st = r.ring + stage * GT_STAGE_BYTES;
        const uint32_t sc = st + (uint32_t)tiles * 1024 + g * 8 + (t >> 1) * 4;
        const int tt0 = c * CT + 4 * wj; // this warp's first tile within the row
        // One tile: the raw code bytes meet the even elements' digits, the
        // high nibbles (x 16) the digits of odd - even; the two halves H of
        // each block pair chain in one accumulator. A lane's columns are two
        // adjacent digits of its block: exact integer sums, combined and
        // scaled in fp32 (two rows per packed instruction).
        auto tile = [&](int i) {
            const int ti = 4 * wj + i;
            const uint32_t tt = (uint32_t)(tt0 + i);
            const uint4 w0 = lds128(st + ti * 1024 + lane * 16);
            const uint4 w1 = lds128(st + ti * 1024 + 512 + lane * 16);
            const uint32_t s0 = lds32(sc + ti * 128), s1 = lds32(sc + ti * 128 + 64);
            const uint4 b0 = lds128(f_base + tt * f_tile);
            const uint4 b1 = lds128(f_base + tt * f_tile + f_pair);
            const float2 bu = lds64f(bs_base + tt * 32);
            constexpr uint32_t HI = 0xF0F0F0F0u;
            int d0[4] = {0, 0, 0, 0}, d1[4] = {0, 0, 0, 0};
            mma_u8s8_16832(d0[0], d0[1], d0[2], d0[3], w0.x, w0.y, w0.x & HI, w0.y & HI, b0.x, b0.y);
            mma_u8s8_16832(d1[0], d1[1], d1[2], d1[3], w1.x, w1.y, w1.x & HI, w1.y & HI, b1.x, b1.y);
            mma_u8s8_16832(d0[0], d0[1], d0[2], d0[3], w0.z, w0.w, w0.z & HI, w0.w & HI, b0.z, b0.w);
            mma_u8s8_16832(d1[0], d1[1], d1[2], d1[3], w1.z, w1.w, w1.z & HI, w1.w & HI, b1.z, b1.w);
            const float2 p0 = make_float2((float)(d0[0] * 128 + d0[1]), (float)(d0[2] * 128 + d0[3]));
            const float2 p1 = make_float2((float)(d1[0] * 128 + d1[1]), (float)(d1[2] * 128 + d1[3]));
            const float2 su0 = mul2_rn(make_float2(decode_scale<AAEDN_SCALE_F16>((uint16_t)(s0 & 0xFFFFu)),
                                                   decode_scale<AAEDN_SCALE_F16>((uint16_t)(s0 >> 16))),
                                       make_float2(bu.x, bu.x));
            const float2 su1 = mul2_rn(make_float2(decode_scale<AAEDN_SCALE_F16>((uint16_t)(s1 & 0xFFFFu)),
                                                   decode_scale<AAEDN_SCALE_F16>((uint16_t)(s1 >> 16))),
                                       make_float2(bu.y, bu.y));
            acc = fma2_rn(p0, su0, acc);
            acc = fma2_rn(p1, su1, acc);
        };
        if (tiles == CT)
        {
#pragma unroll
            for (int i = 0; i < 4; ++i)
                tile(i);
        }
        else
        {
#pragma unroll
            for (int i = 0; i < 4; ++i)
                if (4 * wj + i < tiles)
                    tile(i);
        }
        float acc0 = acc.x, acc1 = acc.y;
        __syncwarp();
        if (lane == 0)
            mbar_arrive(r.empty + 8 * stage);
        if (p.trace && tid == 0)
            trace_chunk(p.trace, cta, qq, 1);
        // the quad's sum (over blocks and digit halves), then this warp's
        // partial of the chunk into its slot
        acc0 += __shfl_xor_sync(0xffffffffu, acc0, 1);
        acc0 += __shfl_xor_sync(0xffffffffu, acc0, 2);
        acc1 += __shfl_xor_sync(0xffffffffu, acc1, 1);
        acc1 += __shfl_xor_sync(0xffffffffu, acc1, 2);
        float* slot = part + ((size_t)(qq % GT_RQ) * GT_GROUP_WARPS + wj) * 16;
        if (t == 0)
        {
            slot[g] = acc0;
            slot[g + 8] = acc1;
        }
        __syncwarp();
        unsigned last = 0;
        if (lane == 0)
        {
            __threadfence_block();
            last = atomicAdd(cnt + (uint32_t)gl % GT_RC, 1u) == (unsigned)(nchunk * GT_GROUP_WARPS) - 1 ? 1u : 0u;
        }
        last = __shfl_sync(0xffffffffu, last, 0);
        if (last)
        {
            // every partial of row group gl is in: sum in fixed order
            // (chunk, warp), then the epilogue on this warp
            __threadfence_block();
            if (lane < 16)
            {
                float s = 0.0f;
                const uint32_t qb = q0 + (uint32_t)(gl * nchunk);
                for (int cc = 0; cc < nchunk; ++cc)
                    for (int w = 0; w < GT_GROUP_WARPS; ++w)
                        s += part[((size_t)((qb + cc) % GT_RQ) * GT_GROUP_WARPS + w) * 16 + lane];
                tmp[lane] = s;
            }
            __syncwarp();
            float post = 1.0f;
            if constexpr (NORM)
            {
                float tss = 0.0f;
                for (int i = 0; i < GT_CONSUMERS; ++i) // fixed order
                    tss += wss[i];
                post = 1.0f / sqrtf(__fadd_rn(__fdiv_rn(tss, (float)p.K), p.eps)); // src/rmsnorm.cpp:34
            }
            gemv_epilogue<1, EPI, 1>(p, tmp, cta + gl * ncta, lane, post, ecp, gl);
            __syncwarp();
            if (lane == 0)
                cnt[(uint32_t)gl % GT_RC] = 0u;
        }
        qq += GT_GROUPS;
        stage += GT_GROUPS;
        while (stage >= NS)
        {
            stage -= NS;
            ++use;
        }
        c += GT_GROUPS;
        while (c >= nchunk)
        {
            c -= nchunk;
            ++gl;
        }
    }
    return !named_bar_or(1, NCT, !ok);
}

// The decode GEMV kernel: one producer warp streaming the CTA's chunks, 24
// consumer warps building the integer operand together, then consuming the
// chunks six at a time.
// At most GT_REGS registers a thread, so that 25 warps fit one CTA (the
// consumers are latency-bound; more warps hide more of it). 80 would be
// 64000 registers, which the launch rejects; 72 leaves headroom.
constexpr int GT_REGS = 72;

template <int PRO, int EPI>
__global__ void __maxnreg__(GT_REGS) gemv_tiled_i8_kernel(const GemvParams p)
{
    const int NS = p.stages > GT_STAGES ? p.stages : GT_STAGES; // the host sizes shared memory so
    constexpr int NC = GT_CONSUMERS;
    constexpr int NCT = NC * 32;
    extern __shared__ __align__(16) uint8_t smem[];
    const int ntile = p.K >> 7;
    uint8_t* ring = smem;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + (size_t)NS * GT_STAGE_BYTES); // full[NS], empty[NS]
    uint8_t* frag = reinterpret_cast<uint8_t*>(bars) + (size_t)NS * 16;
    float* bscale = reinterpret_cast<float*>(frag + (size_t)ntile * GT_FRAG_TILE_BYTES);
    float* red = bscale + (size_t)ntile * 8;
    float* misc = red + GT_RED_BYTES / 4; // GT_MISC_*: per-warp sums of squares, zeros, flags, stage tags
    float* ecache = misc + GT_MISC_FLOATS;
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
    r.tag = smem_addr(misc + GT_MISC_TAG);
    r.ns = (uint32_t)NS;

    if (tid == 0)
    {
        for (int i = 0; i < NS; ++i)
        {
            mbar_init(r.full + 8 * i, 1);
            mbar_init(r.empty + 8 * i, GT_GROUP_WARPS);
            reinterpret_cast<unsigned*>(misc + GT_MISC_TAG)[i] = 0xFFFFFFFFu;
        }
        mbar_init_fence();
        s_abort = 0;
    }
    if (tid < GT_RC)
        reinterpret_cast<unsigned*>(red + GT_RQ * GT_GROUP_WARPS * 16)[tid] = 0u;
    if (tid < 4)
        misc[GT_MISC_ZERO + tid] = 0.0f;
    if (tid == 0)
        reinterpret_cast<unsigned*>(misc)[GT_MISC_FLAG] = 0u;
    __syncthreads();

    if (warp == NC)
    {
        // producer warp: the weights do not depend on the previous kernel
        uint32_t q = 0;
        if (!tiled_produce(p.w, p.N, p.K, r, q, blockIdx.x, gridDim.x, lane, p.l2_hint != 0))
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
    // epilogue inputs for shared memory: loaded into registers first, so
    // their L2 round trip overlaps the operand build's
    constexpr int EPRE = (GT_ECACHE_FLOATS + NCT - 1) / NCT; // per thread
    float epre[EPRE];
    int n_epre = 0;
    if constexpr (EPI == EPI_RESIDUAL)
    {
        const int n_groups = p.N >> 4, cta = blockIdx.x, ncta = gridDim.x;
        const int my_groups = cta < n_groups ? (n_groups - 1 - cta) / ncta + 1 : 0;
        if (my_groups * 16 <= GT_ECACHE_FLOATS)
        {
            n_epre = my_groups * 16;
#pragma unroll
            for (int j = 0; j < EPRE; ++j)
            {
                const int i = tid + j * NCT;
                epre[j] = i < n_epre ? __ldcg(p.y + (size_t)(cta + (i >> 4) * ncta) * 16 + (i & 15)) : 0.0f;
            }
        }
    }
    else if constexpr (EPI == EPI_QKV_ROPE)
    {
        const int half = p.head_dim >> 1;
        const uint32_t pos = p.state->pos;
        if (half <= GT_ECACHE_FLOATS / 2 && pos < (uint32_t)p.max_pos)
        {
            n_epre = 2 * half; // cos at [0, half), sin at [half, 2 half) of the staging order
#pragma unroll
            for (int j = 0; j < EPRE; ++j)
            {
                const int i = tid + j * NCT;
                epre[j] = i < half    ? __ldg(p.rope_cos + (size_t)pos * half + i)
                          : i < n_epre ? __ldg(p.rope_sin + (size_t)pos * half + (i - half))
                                       : 0.0f;
            }
        }
    }
    gt_build<PRO>(p, frag, bscale, misc + GT_MISC_WSS);
#pragma unroll
    for (int j = 0; j < EPRE; ++j)
    {
        const int i = tid + j * NCT;
        if (i < n_epre)
        {
            if constexpr (EPI == EPI_QKV_ROPE)
            {
                const int half = p.head_dim >> 1;
                ecache[i < half ? i : GT_ECACHE_FLOATS / 2 + (i - half)] = epre[j];
            }
            else
                ecache[i] = epre[j];
        }
    }
    named_bar_sync(1, NCT); // the operand and the staged inputs are complete
    if (tid == 0)
        trace_mark(p.trace, blockIdx.x, 1);
    if (!gt_consume<PRO, EPI>(p, r, 0u, frag, bscale, misc + GT_MISC_WSS, smem_addr(misc + GT_MISC_ZERO), red, ecache, blockIdx.x,
                              gridDim.x, s_abort))
    {
        if (lane == 0 && p.state)
            p.state->err = 2u;
    }
    else if (p.tp_sig)
    {
        // tensor parallel: the last CTA to finish copies this rank's partial
        // (complete: every CTA counted itself after a fence) into every other
        // rank's receive buffer, then raises this GEMV's epoch there
        volatile unsigned* last = reinterpret_cast<volatile unsigned*>(misc) + GT_MISC_LAST;
        __threadfence(); // every thread: its rows before the CTA counts itself
        named_bar_sync(1, NCT);
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
        named_bar_sync(1, NCT);
        if (*last)
        {
            const size_t off = ((size_t)p.tpc.rank * 2 + p.tp_buf) * p.tpc.dim;
            const float4* src = reinterpret_cast<const float4*>(p.tpc.recv[p.tpc.rank] + off);
            const int n4 = p.tpc.dim >> 2;
            for (int qq = 0; qq < p.tpc.size; ++qq)
                if (qq != p.tpc.rank)
                {
                    float4* dst = reinterpret_cast<float4*>(p.tpc.recv[qq] + off);
                    for (int i = tid; i < n4; i += NCT)
                        dst[i] = __ldcg(src + i);
                }
            named_bar_sync(1, NCT);
            if (tid == 0)
                tp_signal(p.tpc, *p.tp_epoch + (unsigned)p.tp_sig_phase + 1u); // fences at system scope first
        }
    }
    if (tid == 0)
        trace_mark(p.trace, blockIdx.x, 3);
}

} // namespace aaedn_dev
