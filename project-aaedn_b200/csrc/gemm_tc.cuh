// gemm_tc.cuh — the block-quantized matrix product on the 5th-generation
// tensor cores (tcgen05.mma, accumulators in tensor memory), for more than
// eight activation rows: prefill and the fused_matmul API at M > 8.
//
// Replaces the intended product of src/fused_matmul.cpp:70-169 (out[m][n] =
// sum_k in[m][k] * code(n, k) * scale(n, k / 32)) for many rows at once.
//
// Roles: D[n][m] = sum_k W[n][k] * X[m][k], with the weights as the MMA's A
// operand (128 weight rows per CTA tile, UMMA M = 128) and the activations
// as B (BN activation rows per tile, UMMA N = BN); the fp32 accumulator tile
// [128 lanes = weight rows][BN columns = activation rows] lives in TMEM.
//
// Precision: the MMA takes bf16 operands. A dequantized weight code * scale
// (a 4-bit integer times an fp16 value: at most 15 significant bits) is
// exactly w_hi + w_lo with both parts bf16; the fp32 activation is split into
// three bf16 parts x_hi + x_mid + x_lo (24 significant bits, what fp32
// carries). The accumulator receives the five products whose magnitude is
// above 2^-24 of the leading one (x_hi w_hi, x_mid w_hi, x_lo w_hi, x_hi w_lo,
// x_mid w_lo), so the product is fp32-accurate: the tensor pipe does 5 bf16
// MMAs per fp32 multiply-add of the product. The tensor core rounds each
// MMA's sum into its accumulator with an error of up to one unit in the last
// place of the accumulator, so the four small products go to a second
// accumulator (2^-8 of the first's magnitude): the leading accumulator takes
// K / 16 additions instead of 5 K / 16; the epilogue adds the two in fp32.
//
// Data movement, per stage of 64 K:
//   * the activation parts (prepared once per call in global memory as bf16
//     [3][M_pad][K], K in the tc_kpos order) arrive by TMA
//     (cp.async.bulk.tensor, 128-byte swizzle: the canonical K-major layout
//     the MMA reads), issued by warp 8;
//   * the weights' 4-bit codes and fp16 scales are read from global memory by
//     warps 0-7 (two threads per weight row, one quant block of 16 bytes
//     each per stage, loaded two stages ahead), dequantized in registers
//     (bf16x2 and packed fp32 arithmetic, exact) and written as the two bf16
//     parts into the same swizzled layout (fence.proxy.async before the
//     stage is marked full);
//   * warp 9 issues the 20 MMAs of the stage (4 k-steps x 5 part products)
//     from one thread and commits them to the stage's "empty" barrier.
// Epilogue: warps w and w + 4 read TMEM lanes 32 (w % 4).. (tcgen05.ld
// 32x32b), half of the columns each, and store out[m][n] (a warp writes 32
// consecutive n of one m: coalesced).
//
// Every wait is bounded (globaltimer): a wait that runs out sets *err, the
// kernel drains what it issued, frees its TMEM and returns.
#pragma once

#include <cuda.h> // CUtensorMap

#include "common.cuh"
#include "gemm_tc.h"

namespace aaedn_dev
{

constexpr int TC_BM = 128;     // weight rows per tile (UMMA M)
constexpr int TC_BK = 64;      // K per stage: one 128-byte swizzle row of bf16
constexpr int TC_XP = 3;       // bf16 parts of the activation
constexpr int TC_WP = 2;       // bf16 parts of a dequantized weight (exact)
constexpr int TC_DQ_WARPS = 8;  // dequant + epilogue warps (two threads per weight row)
constexpr int TC_TMA_WARP = TC_DQ_WARPS, TC_MMA_WARP = TC_DQ_WARPS + 1;
constexpr int TC_THREADS = (TC_DQ_WARPS + 2) * 32;
constexpr uint64_t TC_WAIT_LIMIT_NS = 2000000000ull;

struct TcGemmParams
{
    const uint8_t* w;  // codes (and, tiled, scales)
    const uint16_t* s; // row-major scales
    size_t ldb;        // row-major: codes per weight row
    int w_layout;
    int N, K, M;       // weight rows, reduction length, activation rows
    int k_per_split;   // K handled by the CTAs of one blockIdx.z (a multiple of 64)
    float* out;        // blockIdx.z == s writes out + s * split_stride
    size_t ldc, split_stride;
    unsigned* err;     // set to 1 when a bounded wait ran out
    TcEpi e;           // the model's epilogues
};

template <int BN, int STAGES>
struct TcSmem
{
    static constexpr size_t W_PART = (size_t)TC_BM * 128; // 16 KB
    static constexpr size_t X_PART = (size_t)BN * 128;
    static constexpr size_t STAGE = TC_WP * W_PART + TC_XP * X_PART;
    static constexpr size_t BARS = 1024; // after the stages: mbarriers, TMEM address
    static constexpr size_t BYTES = STAGES * STAGE + BARS + 1024; // + alignment slack
    static_assert(BYTES <= 232448, "GEMM stages exceed the shared memory of a CTA");
    static constexpr uint32_t TMEM_COLS = 2 * BN; // leading + small-product accumulators (a power of two)
};

// ---- tcgen05 / TMA primitives ----------------------------------------------
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row groups
// 1024 bytes apart (SBO), leading offset unused (16 B), sm100 version 1.
__device__ __forceinline__ uint64_t tc_desc_sw128(uint32_t saddr)
{
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1u << 16) | ((uint64_t)(1024u >> 4) << 32) |
           ((uint64_t)1u << 46) | ((uint64_t)2u << 61);
}

// Instruction descriptor of kind::f16: bf16 A and B, fp32 D, both K-major,
// M = 128, N = n.
__host__ __device__ constexpr uint32_t tc_idesc_bf16(int n)
{
    return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(TC_BM >> 4) << 24);
}

__device__ __forceinline__ void tc_mma(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t acc)
{
    asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                 "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
                 "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc)
                 : "memory");
}

// Arrives once on the mbarrier when every MMA this thread issued so far is done.
__device__ __forceinline__ void tc_commit(uint32_t mbar)
{
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(mbar)
                 : "memory");
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const void* tmap, int x, int y, uint32_t mbar)
{
    asm volatile("cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
                 "[%4];" ::"r"(dst),
                 "l"(tmap), "r"(x), "r"(y), "r"(mbar)
                 : "memory");
}

__device__ __forceinline__ void tc_ld8(uint32_t taddr, float (&v)[8])
{
    uint32_t r[8];
    // one statement: the registers are read only after the wait
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];\n\t"
                 "tcgen05.wait::ld.sync.aligned;"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr)
                 : "memory");
#pragma unroll
    for (int i = 0; i < 8; ++i)
        v[i] = __uint_as_float(r[i]);
}

// 16 bytes of codes (32 weights of one quant block) dequantized with scale
// sc into their two bf16 parts, stored as the 16-byte chunks c0..c0+3 of a
// 128-byte swizzled row (chunk c at (c ^ r7) * 16). Exact: code * scale has
// at most 15 significant bits, w_hi = bf16(w) and w_lo = w - w_hi.
__device__ __forceinline__ void tc_dequant_block(uint4 codes, float sc, uint32_t w0_row, uint32_t w1_row, int c0,
                                                 uint32_t r7)
{
    const uint32_t cw[4] = {codes.x, codes.y, codes.z, codes.w};
    const float2 sc2 = make_float2(sc, sc);
    const float2 neg1 = make_float2(-1.0f, -1.0f);
#pragma unroll
    for (int j = 0; j < 4; ++j)
    {
        uint32_t hi[4], lo[4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
        {
            // codes i and i + 4 of the word as bf16 (128 + c) - 128: exact
            uint32_t cp = ((cw[j] >> (4 * i)) & 0x000F000Fu) | 0x43004300u;
            asm("sub.rn.bf16x2 %0, %0, %1;" : "+r"(cp) : "r"(0x43004300u));
            const float2 c = make_float2(__uint_as_float(cp << 16), __uint_as_float(cp & 0xFFFF0000u));
            const float2 w = mul2_rn(c, sc2); // exact
            const __nv_bfloat162 h = __floats2bfloat162_rn(w.x, w.y);
            const uint32_t hu = *reinterpret_cast<const uint32_t*>(&h);
            const float2 hf = make_float2(__uint_as_float(hu << 16), __uint_as_float(hu & 0xFFFF0000u));
            const float2 r = fma2_rn(hf, neg1, w); // w - w_hi, exact
            const __nv_bfloat162 l = __floats2bfloat162_rn(r.x, r.y);
            hi[i] = hu;
            lo[i] = *reinterpret_cast<const uint32_t*>(&l);
        }
        const uint32_t chunk = (((uint32_t)(c0 + j)) ^ r7) * 16u;
        asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(w0_row + chunk), "r"(hi[0]), "r"(hi[1]),
                     "r"(hi[2]), "r"(hi[3])
                     : "memory");
        asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(w1_row + chunk), "r"(lo[0]), "r"(lo[1]),
                     "r"(lo[2]), "r"(lo[3])
                     : "memory");
    }
}

// The 16 code bytes of quant block b of weight row `row` and its fp16 scale.
__device__ __forceinline__ void tc_w_load(const TcGemmParams& p, int row, int b, uint4& ca, uint16_t& sc)
{
    if (p.w_layout == TC_W_TILED)
    {
        // the decode GEMV's layout (gemv_tiled.cuh): chunks of 16 tiles;
        // block b is half b' = b % 2 of pair P = (b % 4) / 2 of its tile,
        // whose code bytes for rows g and g + 8 sit in lanes 4g..4g+3: word
        // (H, r) of lane 4g + t = bytes [8H + 4(t & 1), +4) of block
        // 2P + (t >> 1)
        constexpr int CT = 16;
        const int ntile = p.K >> 7, group = row >> 4, r16 = row & 15, r = r16 >> 3, g = r16 & 7;
        const int tile = b >> 2, P = (b >> 1) & 1, bp = b & 1, c = tile / CT, ti = tile % CT;
        const int tiles_in_chunk = min(CT, ntile - CT * c);
        const uint8_t* chunk = p.w + (size_t)group * ntile * 1152 + (size_t)c * CT * 1152;
        // lane 4g + 2b' + h: words (H0 r0, H0 r1, H1 r0, H1 r1)
        const uint32_t* q = reinterpret_cast<const uint32_t*>(chunk + (size_t)ti * 1024 + P * 512 +
                                                              (4 * g + 2 * bp) * 16);
        ca = make_uint4(__ldg(q + r), __ldg(q + 4 + r), __ldg(q + 2 + r), __ldg(q + 6 + r));
        sc = __ldg(reinterpret_cast<const uint16_t*>(chunk + (size_t)tiles_in_chunk * 1024 + ti * 128) +
                   ((P * 8 + g) * 2 + bp) * 2 + r);
    }
    else
    {
        ca = __ldg(reinterpret_cast<const uint4*>(p.w + (size_t)row * (p.ldb >> 1) + (size_t)b * 16));
        sc = __ldg(p.s + (size_t)row * (p.ldb >> 5) + b);
    }
}

// The paired epilogues for one activation row m: v = D[rbase + jj][m] and
// u = D[rbase + 8 + jj][m] (jj < 8) of the 16-row group at rbase.
//   SWIGLU: act[m][rbase / 2 + jj] = silu(v) * u (gate and up rows
//           interleaved in 8-row chunks)
//   QKV:    q and k rows: the rotate-half pair (i, i + hd/2) sits in rows
//           (jj, jj + 8) of the group; RoPE at the row's position, q to
//           qrows, k (and v, unrotated) appended to the row's page.
template <int EPI>
__device__ __forceinline__ void tc_pair_epilogue(const TcEpi& e, int m, int rbase, int jj, float v, float u)
{
    if constexpr (EPI == TC_EPI_SWIGLU)
        e.act[(size_t)m * e.ld_act + (rbase >> 1) + jj] = __fmul_rn(silu_f(v), u); // D6
    else
    {
        const int hd = e.head_dim, half = hd >> 1;
        const bool isq = rbase < e.q_rows, isk = !isq && rbase < e.q_rows + e.kv_rows;
        const int rel = isq ? rbase : (isk ? rbase - e.q_rows : rbase - e.q_rows - e.kv_rows);
        const int h = rel / hd;
        const int i = ((rel % hd) >> 4) * 8 + jj; // rope pair (i, i + half)
        const int pos = e.row_pos ? e.row_pos[m] : e.pos0 + m;
        const int* pt = e.row_seq ? e.page_table + (size_t)e.row_seq[m] * e.pt_stride : e.page_table;
        const int page = pt[pos / e.page_size], slot = pos % e.page_size;
        float* kv = nullptr;
        if (!isq)
            kv = (isk ? e.k_layer : e.v_layer) + (((size_t)page * e.n_kv + h) * e.page_size + slot) * hd;
        if (isq || isk)
        {
            // rotate-half at the absolute position (D3, src/rope.cpp:53-54)
            const float c = e.rope_cos[(size_t)pos * half + i], sn = e.rope_sin[(size_t)pos * half + i];
            const float o0 = __fsub_rn(__fmul_rn(c, v), __fmul_rn(sn, u));
            const float o1 = __fadd_rn(__fmul_rn(sn, v), __fmul_rn(c, u));
            float* dst = isq ? e.qrows + (size_t)m * e.ldq + (size_t)h * hd : kv;
            dst[i] = o0;
            dst[i + half] = o1;
        }
        else
        {
            const int d = rel % hd + jj;
            kv[d] = v;
            kv[d + 8] = u;
        }
    }
}

// Epilogue of 8 activation rows (columns c0.. of the accumulator) of weight
// row `row` (thread = TMEM lane), values v. Every lane of the warp calls it
// (the paired epilogues exchange values between lanes r and r + 8).
template <int EPI>
__device__ __forceinline__ void tc_epilogue8(const TcGemmParams& p, float* out, int row, bool live, int m_first,
                                             const float (&v)[8])
{
    if constexpr (EPI == TC_EPI_STORE || EPI == TC_EPI_RESID)
    {
        if (!live)
            return;
#pragma unroll
        for (int j = 0; j < 8; ++j)
        {
            const int m = m_first + j;
            if (m < p.M)
            {
                float* o = out + (size_t)m * p.ldc + row;
                if constexpr (EPI == TC_EPI_STORE)
                    *o = v[j];
                else
                    *o = v[j] + *o; // src/transformer.cpp:214, 227 (tmp + hidden)
            }
        }
    }
    else
    {
        float u[8];
#pragma unroll
        for (int j = 0; j < 8; ++j)
            u[j] = __shfl_down_sync(0xffffffffu, v[j], 8); // row + 8 of the same 16-row group
        const int jj = row & 15, rbase = row & ~15;
        if (!live || jj >= 8)
            return;
#pragma unroll
        for (int j = 0; j < 8; ++j)
        {
            const int m = m_first + j;
            if (m < p.M)
                tc_pair_epilogue<EPI>(p.e, m, rbase, jj, v[j], u[j]);
        }
    }
}

template <int BN, int STAGES, int EPI>
__global__ void __launch_bounds__(TC_THREADS, 1) q4_gemm_tc_kernel(const TcGemmParams p,
                                                                    const __grid_constant__ CUtensorMap xmap)
{
    using SM = TcSmem<BN, STAGES>;
    extern __shared__ __align__(16) uint8_t smem_raw[];
    // 1024-byte alignment: the 128-byte swizzle pattern is taken from address bits
    const uint32_t raw_a = smem_addr(smem_raw);
    const uint32_t base = (raw_a + 1023u) & ~1023u;
    const uint32_t bar0 = base + (uint32_t)(STAGES * SM::STAGE);
    // barriers: full_x[S], full_w[S], empty[S], accum; then the TMEM address
    auto full_x = [&](int s) { return bar0 + 8u * s; };
    auto full_w = [&](int s) { return bar0 + 8u * (STAGES + s); };
    auto empty = [&](int s) { return bar0 + 8u * (2 * STAGES + s); };
    const uint32_t accum = bar0 + 8u * (3 * STAGES);
    const uint32_t tmem_slot = bar0 + 8u * (3 * STAGES + 1);
    __shared__ int s_abort_mem;
    volatile int& s_abort = s_abort_mem;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int n0 = blockIdx.x * TC_BM, m0 = blockIdx.y * BN;
    const int kb0 = blockIdx.z * (p.k_per_split / TC_BK); // first 64-wide K block of this CTA
    const int nk = min(p.K - blockIdx.z * p.k_per_split, p.k_per_split) / TC_BK;
    float* out = p.out + (size_t)blockIdx.z * p.split_stride;
    const uint32_t M_pad = (uint32_t)((p.M + BN - 1) / BN * BN);

    if (tid == 0)
    {
        for (int s = 0; s < STAGES; ++s)
        {
            mbar_init(full_x(s), 1);
            mbar_init(full_w(s), TC_DQ_WARPS * 32);
            mbar_init(empty(s), 1);
        }
        mbar_init(accum, 1);
        mbar_init_fence();
        s_abort = 0;
    }
    if (warp == TC_MMA_WARP)
    {
        // two accumulators of BN fp32 columns
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(tmem_slot),
                     "r"(SM::TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = lds32(tmem_slot);

    auto w_part = [&](int s, int j) { return base + (uint32_t)(s * SM::STAGE + j * SM::W_PART); };
    auto x_part = [&](int s, int i) { return base + (uint32_t)(s * SM::STAGE + TC_WP * SM::W_PART + i * SM::X_PART); };
    auto fail = [&]() {
        s_abort = 1;
        if (p.err)
            atomicExch(p.err, 1u);
    };

    if (warp == TC_TMA_WARP)
    {
        // ---- TMA producer of the activation parts
        int issued = 0;
        if (lane == 0)
        {
            for (int kb = 0; kb < nk; ++kb)
            {
                const int s = kb % STAGES, use = kb / STAGES;
                if (use > 0 && !mbar_wait_bounded(empty(s), (use - 1) & 1, TC_WAIT_LIMIT_NS))
                {
                    fail();
                    break;
                }
                if (s_abort)
                    break;
                mbar_arrive_expect_tx(full_x(s), (uint32_t)(TC_XP * SM::X_PART));
                for (int i = 0; i < TC_XP; ++i)
                    tma_load_2d(x_part(s, i), &xmap, (kb0 + kb) * TC_BK, (int)(i * M_pad) + m0, full_x(s));
                ++issued;
            }
            // the copies it issued have landed before the CTA may exit
            for (int kb = issued > STAGES ? issued - STAGES : 0; kb < issued; ++kb)
                mbar_wait_bounded(full_x(kb % STAGES), (kb / STAGES) & 1, TC_WAIT_LIMIT_NS);
        }
        __syncwarp();
    }
    else if (warp == TC_MMA_WARP)
    {
        // ---- MMA issuer (one thread)
        if (lane == 0)
        {
            constexpr uint32_t idesc = tc_idesc_bf16(BN);
            // (x part, w part) products, largest first
            const int px[5] = {0, 1, 0, 2, 1}, pw[5] = {0, 0, 1, 0, 1};
            bool ok = true;
            for (int kb = 0; kb < nk && ok; ++kb)
            {
                const int s = kb % STAGES;
                const uint32_t ph = (uint32_t)(kb / STAGES) & 1;
                if (!mbar_wait_bounded(full_x(s), ph, TC_WAIT_LIMIT_NS) ||
                    !mbar_wait_bounded(full_w(s), ph, TC_WAIT_LIMIT_NS) || s_abort)
                {
                    fail();
                    ok = false;
                    break;
                }
                tc_fence_after();
#pragma unroll
                for (int k = 0; k < TC_BK / 16; ++k)
#pragma unroll
                    for (int q = 0; q < 5; ++q)
                        // q = 0 into columns [0, BN), the rest into [BN, 2 BN); the first
                        // product into each overwrites it
                        tc_mma(tmem + (q ? (uint32_t)BN : 0u), tc_desc_sw128(w_part(s, pw[q]) + k * 32),
                               tc_desc_sw128(x_part(s, px[q]) + k * 32), idesc,
                               (kb | k | (q > 1 ? 1 : 0)) != 0 ? 1u : 0u);
                tc_commit(empty(s)); // the stage's smem is free once these MMAs are done
            }
            // always: the epilogue (and the TMEM release) waits for every MMA
            // issued, on success or not
            tc_commit(accum);
        }
        __syncwarp();
    }
    else
    {
        // ---- warps 0-7: thread (half h, row r) = (tid / 128, tid % 128)
        // dequantizes quant block h of the stage's 64 K of weight row n0 + r
        const int r = tid & 127, h = tid >> 7;
        const int row = n0 + r;
        const bool live = row < p.N;
        const uint32_t r7 = (uint32_t)(r & 7);
        // registers two stages ahead: slot A for even kb, slot B for odd
        uint4 cwa = make_uint4(0, 0, 0, 0), cwb = make_uint4(0, 0, 0, 0);
        uint16_t sca = 0, scb = 0;
        auto load = [&](int kb, uint4& cw, uint16_t& sc) {
            if (live && kb < nk)
                tc_w_load(p, row, (kb0 + kb) * 2 + h, cw, sc);
            else
            {
                cw = make_uint4(0, 0, 0, 0);
                sc = 0;
            }
        };
        // one stage: false when a wait ran out or the CTA aborts
        auto stage = [&](int kb, uint4& cw, uint16_t& sc) -> bool {
            const int s = kb % STAGES, use = kb / STAGES;
            if (use > 0 && !mbar_wait_bounded(empty(s), (use - 1) & 1, TC_WAIT_LIMIT_NS))
            {
                fail();
                return false;
            }
            if (s_abort)
                return false;
            const uint32_t w0 = w_part(s, 0) + (uint32_t)r * 128, w1 = w_part(s, 1) + (uint32_t)r * 128;
            tc_dequant_block(cw, __half2float(__ushort_as_half(sc)), w0, w1, 4 * h, r7);
            load(kb + 2, cw, sc);
            // generic-proxy stores, then visible to the tensor core's reads
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            mbar_arrive(full_w(s));
            return true;
        };
        load(0, cwa, sca);
        load(1, cwb, scb);
        for (int kb = 0; kb < nk; kb += 2)
            if (!stage(kb, cwa, sca) || (kb + 1 < nk && !stage(kb + 1, cwb, scb)))
                break;
        // ---- epilogue: TMEM lanes 32 (warp % 4) + lane = weight rows, the
        // warp's half (warp / 4) of the BN activation columns
        if (mbar_wait_bounded(accum, 0, TC_WAIT_LIMIT_NS) && !s_abort)
        {
            tc_fence_after();
            const int erow = n0 + 32 * (warp & 3) + lane;
            const uint32_t t_row = tmem + ((uint32_t)((warp & 3) * 32) << 16);
            const int cbeg = (warp >> 2) * (BN / 2);
            for (int c0 = cbeg; c0 < cbeg + BN / 2; c0 += 8)
            {
                float v[8], w[8];
                tc_ld8(t_row + (uint32_t)c0, v);
                tc_ld8(t_row + (uint32_t)(BN + c0), w);
#pragma unroll
                for (int j = 0; j < 8; ++j)
                    v[j] += w[j];
                tc_epilogue8<EPI>(p, out, erow, erow < p.N, m0 + c0, v);
            }
        }
        else
            fail();
    }
    tc_fence_before();
    __syncthreads();
    if (warp == TC_MMA_WARP)
    {
        // every MMA issued has completed before its accumulator is released
        if (lane == 0)
            mbar_wait_bounded(accum, 0, TC_WAIT_LIMIT_NS);
        __syncwarp();
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(SM::TMEM_COLS)
                     : "memory");
    }
}

// Splits fp32 activation rows into the three bf16 parts the GEMM reads:
// parts[i][m][tc_kpos(k)] for m < M_pad (rows M..M_pad-1 zero); 8 elements
// (one group of the K order) per thread.
__global__ void tc_split_kernel(const float* __restrict__ x, size_t lda, int M, int M_pad, int K,
                                __nv_bfloat16* __restrict__ parts)
{
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    const size_t per_row = (size_t)K / 8;
    if (i >= (size_t)M_pad * per_row)
        return;
    const int m = (int)(i / per_row), k = (int)(i - (size_t)m * per_row) * 8;
    float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (m < M)
    {
        const float* src = x + (size_t)m * lda + k;
#pragma unroll
        for (int j = 0; j < 8; ++j)
            v[j] = src[j];
    }
    __nv_bfloat16 h[3][8];
#pragma unroll
    for (int j = 0; j < 8; ++j)
    {
        const int q = tc_kpos(j);
        h[0][q] = __float2bfloat16_rn(v[j]);
        const float r1 = v[j] - __bfloat162float(h[0][q]);
        h[1][q] = __float2bfloat16_rn(r1);
        h[2][q] = __float2bfloat16_rn(r1 - __bfloat162float(h[1][q]));
    }
    const size_t plane = (size_t)M_pad * K;
#pragma unroll
    for (int q = 0; q < 3; ++q)
    {
        uint4 w;
        w.x = pack_bf16(h[q][0], h[q][1]);
        w.y = pack_bf16(h[q][2], h[q][3]);
        w.z = pack_bf16(h[q][4], h[q][5]);
        w.w = pack_bf16(h[q][6], h[q][7]);
        *reinterpret_cast<uint4*>(parts + q * plane + (size_t)m * K + k) = w;
    }
}

// The split-K sum for the paired epilogues: one thread per (activation row
// m, 16-row group, jj < 8) adds the splits of rows rbase + jj and
// rbase + 8 + jj in order and applies the epilogue.
template <int EPI>
__global__ void tc_splitk_pair_kernel(const float* __restrict__ part, int splits, size_t split_stride, int M, int N,
                                      const TcEpi e)
{
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    const size_t per_m = (size_t)(N / 16) * 8;
    if (i >= (size_t)M * per_m)
        return;
    const int m = (int)(i / per_m), r = (int)(i - (size_t)m * per_m);
    const int rbase = (r >> 3) * 16, jj = r & 7;
    float v = 0.0f, u = 0.0f;
    for (int s = 0; s < splits; ++s)
    {
        const float* ps = part + (size_t)s * split_stride + (size_t)m * N + rbase + jj;
        v += ps[0];
        u += ps[8];
    }
    tc_pair_epilogue<EPI>(e, m, rbase, jj, v, u);
}

// out[m][n] = (accumulate ? out[m][n] : 0) + the sum over s of part[s][m][n]
// (splits summed in order: deterministic).
__global__ void tc_splitk_reduce_kernel(const float* __restrict__ part, int splits, size_t split_stride, int M, int N,
                                        float* __restrict__ out, size_t ldc, int accumulate)
{
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (size_t)M * N)
        return;
    const int m = (int)(i / N), n = (int)(i - (size_t)m * N);
    float v = 0.0f;
    for (int s = 0; s < splits; ++s)
        v += part[(size_t)s * split_stride + (size_t)m * N + n];
    float* o = out + (size_t)m * ldc + n;
    *o = accumulate ? v + *o : v;
}

} // namespace aaedn_dev
