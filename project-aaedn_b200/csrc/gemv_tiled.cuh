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

} // namespace aaedn_dev
