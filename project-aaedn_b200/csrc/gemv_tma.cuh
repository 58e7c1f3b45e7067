// gemv_tma.cuh — the decode dequant-GEMV with a TMA-fed shared-memory ring.
//
// Same arithmetic as gemv_q4.cuh (codes -> bf16 16+c, tensor-core dot
// products against the bf16 hi/lo split of the activations, per-block scale
// and bias removal in fp32), but the weights move by bulk asynchronous copies
// (cp.async.bulk, the TMA engine) instead of per-thread copies:
//  * one producer warp walks the CTA's work in order and, per chunk of 16
//    rows x 2048 codes, issues 32 bulk copies in one warp instruction (lane l
//    < 16: the 1024 code bytes of row l; lane l >= 16: the 128 scale bytes of
//    row l-16) that complete on the chunk's "full" mbarrier;
//  * the 8 consumer warps share every chunk (warp w takes tiles w and w+8 of
//    its 16 tiles of 128 codes), wait on "full", compute from shared memory
//    and release the slot on its "empty" mbarrier; the producer runs up to
//    GEMV_TMA_STAGES chunks ahead, across row groups, and starts before the
//    activation prologue (and, with programmatic dependent launch, before the
//    previous kernel has ended).
// Requirements (checked by the host): N % 16 == 0, K % 256 == 0, ldb % 256
// == 0, 16-byte aligned weights and scales, an even first tile.
#pragma once

#include "gemv_q4.cuh"

namespace aaedn_dev
{

constexpr int GEMV_TMA_CONSUMERS = 16; // one tile of every 16-tile chunk per warp
constexpr int GEMV_TMA_THREADS = (GEMV_TMA_CONSUMERS + 1) * 32;
constexpr int GEMV_TMA_STAGES = 4;
constexpr int GEMV_TMA_CHUNK_TILES = 16;                           // 2048 codes
constexpr int GEMV_TMA_ROW_BYTES = GEMV_TMA_CHUNK_TILES * 64;      // 1024
constexpr int GEMV_TMA_ROW_STRIDE = GEMV_TMA_ROW_BYTES + 16;       // padded: rows g, g+1 on different banks
constexpr int GEMV_TMA_CODE_BYTES = 16 * GEMV_TMA_ROW_STRIDE;      // 16640
constexpr int GEMV_TMA_SROW_BYTES = GEMV_TMA_CHUNK_TILES * 8;      // 64 scales = 128 B per row
constexpr int GEMV_TMA_STAGE_BYTES = GEMV_TMA_CODE_BYTES + 16 * GEMV_TMA_SROW_BYTES;
constexpr uint64_t GEMV_WAIT_LIMIT_NS = 2000000000ull; // 2 s

inline size_t gemv_tma_smem_bytes(int ntile)
{
    return (size_t)GEMV_TMA_STAGES * GEMV_TMA_STAGE_BYTES + (size_t)GEMV_TMA_STAGES * 16 +
           (size_t)(ntile + 1) * 512 + (size_t)ntile * 16 + (size_t)2 * GEMV_TMA_CONSUMERS * 16 * 4 + 64 * 4;
}

// Scaled, bias-corrected partial sums of rows g and g+8 over tiles i0 and
// (when has1) i1 of a staged chunk: r0[k] / r1[k] is the contribution of
// tile k for row g / g+8.
__device__ __forceinline__ void tile_pair_dot(uint32_t st, uint32_t w_off0, uint32_t w_off1, uint32_t s_off0,
                                              uint32_t s_off1, uint32_t sh, uint32_t f_base, uint32_t f_step,
                                              uint32_t tb_base, int tile0, int i0, int i1, bool has1, float r0[2],
                                              float r1[2])
{
    const int ii[2] = {i0, i1};
    uint4 wa4[2], wb4[2];
    float sc0[2], sc1[2], tbv[2];
    uint32_t fa[2];
#pragma unroll
    for (int k = 0; k < 2; ++k)
    {
        const int i = (k == 0 || has1) ? ii[k] : ii[0];
        wa4[k] = lds128(st + w_off0 + i * 64);
        wb4[k] = lds128(st + w_off1 + i * 64);
        const uint32_t sp = lds32(st + s_off0 + i * 8), sq = lds32(st + s_off1 + i * 8);
        sc0[k] = decode_scale<AAEDN_SCALE_F16>((uint16_t)(sp >> sh));
        sc1[k] = decode_scale<AAEDN_SCALE_F16>((uint16_t)(sq >> sh));
        fa[k] = f_base + (uint32_t)(tile0 + i) * f_step;
        tbv[k] = ldsf(tb_base + (uint32_t)(tile0 + i) * 16);
    }
    float d[2][2][4]; // [tile][even/odd k-step][accumulator]
#pragma unroll
    for (int k = 0; k < 2; ++k)
#pragma unroll
        for (int e = 0; e < 2; ++e)
#pragma unroll
            for (int j = 0; j < 4; ++j)
                d[k][e][j] = 0.0f;
#pragma unroll
    for (int qq = 0; qq < 4; ++qq)
    {
#pragma unroll
        for (int k = 0; k < 2; ++k)
        {
            const uint32_t wa = u4get(wa4[k], qq), wb = u4get(wb4[k], qq);
            const uint4 b = lds128(fa[k] + qq * 128);
            float* dd = d[k][qq & 1];
            mma_bf16_16816(dd[0], dd[1], dd[2], dd[3], nib_e0(wa), nib_e0(wb), nib_e1(wa), nib_e1(wb), b.x, b.y);
            mma_bf16_16816(dd[0], dd[1], dd[2], dd[3], nib_e2(wa), nib_e2(wb), nib_e3(wa), nib_e3(wb), b.z, b.w);
        }
    }
#pragma unroll
    for (int k = 0; k < 2; ++k)
    {
        const float s0 = (d[k][0][0] + d[k][1][0]) + (d[k][0][1] + d[k][1][1]);
        const float s1 = (d[k][0][2] + d[k][1][2]) + (d[k][0][3] + d[k][1][3]);
        r0[k] = (k == 0 || has1) ? sc0[k] * (s0 - tbv[k]) : 0.0f;
        r1[k] = (k == 0 || has1) ? sc1[k] * (s1 - tbv[k]) : 0.0f;
    }
}

template <int PRO, int EPI>
__global__ void __launch_bounds__(GEMV_TMA_THREADS, 1) gemv_tma_kernel(const GemvParams p)
{
    constexpr int NS = GEMV_TMA_STAGES;
    constexpr int NC = GEMV_TMA_CONSUMERS;
    constexpr int NCT = NC * 32;
    constexpr int CT = GEMV_TMA_CHUNK_TILES;
    extern __shared__ __align__(16) uint8_t smem[];
    const int ntile = p.kt1 - p.kt0;
    const int nchunk = (ntile + CT - 1) / CT; // per row group; the last one may be short
    uint8_t* ring = smem;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + (size_t)NS * GEMV_TMA_STAGE_BYTES); // full[NS], empty[NS]
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
        // ---------------- producer warp ----------------
        const size_t wrow = p.ldb >> 1, srow = p.ldb >> 5;
        uint32_t q = 0;
        bool ok = true;
        for (int gl = 0; gl < my_groups && ok; ++gl)
        {
            const int row_l = (blockIdx.x + gl * gridDim.x) * 16 + (lane & 15);
            const uint8_t* wr = p.w + (size_t)row_l * wrow + (size_t)p.kt0 * 64;
            const uint16_t* sr = p.s + (size_t)row_l * srow + (size_t)p.kt0 * 4;
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
                    mbar_arrive_expect_tx(full_a + 8 * stage, (uint32_t)tiles * (16 * 64 + 16 * 8));
                __syncwarp();
                const uint32_t st = ring_a + stage * GEMV_TMA_STAGE_BYTES;
                if (lane < 16)
                    bulk_g2s(st + lane * GEMV_TMA_ROW_STRIDE, wr + (size_t)c * GEMV_TMA_ROW_BYTES, tiles * 64u,
                             full_a + 8 * stage);
                else
                    bulk_g2s(st + GEMV_TMA_CODE_BYTES + (lane - 16) * GEMV_TMA_SROW_BYTES,
                             sr + (size_t)c * (CT * 4), tiles * 8u, full_a + 8 * stage);
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
    const uint32_t w_off0 = (uint32_t)g * GEMV_TMA_ROW_STRIDE + (uint32_t)t * 16;
    const uint32_t w_off1 = w_off0 + 8 * GEMV_TMA_ROW_STRIDE;
    // scale of block 4i + t of rows g / g+8 (read as the aligned u32 pair)
    const uint32_t s_off0 = GEMV_TMA_CODE_BYTES + (uint32_t)g * GEMV_TMA_SROW_BYTES + (uint32_t)(t & 2) * 2;
    const uint32_t s_off1 = s_off0 + 8 * GEMV_TMA_SROW_BYTES;
    const uint32_t sh = (t & 1) * 16;
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
            const uint32_t st = ring_a + stage * GEMV_TMA_STAGE_BYTES;
            // tile `warp` of the chunk: two independent accumulator chains
            // (even / odd k-steps)
            if (warp < tiles)
            {
                const int i = warp, tt = c * CT + i;
                const uint4 wa4 = lds128(st + w_off0 + i * 64);
                const uint4 wb4 = lds128(st + w_off1 + i * 64);
                const uint32_t sp = lds32(st + s_off0 + i * 8), sq = lds32(st + s_off1 + i * 8);
                const uint32_t fa = f_base + (uint32_t)tt * f_step;
                float d[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
                for (int qq = 0; qq < 4; ++qq)
                {
                    const uint32_t wa = u4get(wa4, qq), wb = u4get(wb4, qq);
                    const uint4 b = lds128(fa + qq * 128);
                    float* dd = d[qq & 1];
                    mma_bf16_16816(dd[0], dd[1], dd[2], dd[3], nib_e0(wa), nib_e0(wb), nib_e1(wa), nib_e1(wb), b.x,
                                   b.y);
                    mma_bf16_16816(dd[0], dd[1], dd[2], dd[3], nib_e2(wa), nib_e2(wb), nib_e3(wa), nib_e3(wb), b.z,
                                   b.w);
                }
                const float tbv = ldsf(tb_base + (uint32_t)tt * 16);
                const float sc0 = decode_scale<AAEDN_SCALE_F16>((uint16_t)(sp >> sh));
                const float sc1 = decode_scale<AAEDN_SCALE_F16>((uint16_t)(sq >> sh));
                acc0 = fmaf(sc0, ((d[0][0] + d[1][0]) + (d[0][1] + d[1][1])) - tbv, acc0);
                acc1 = fmaf(sc1, ((d[0][2] + d[1][2]) + (d[0][3] + d[1][3])) - tbv, acc1);
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
