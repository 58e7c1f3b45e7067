// mega.cuh — one decode step as ONE persistent kernel.
//
// A launch of one CTA per SM (cooperative: all CTAs resident) runs every
// phase of the step, separated by grid barriers instead of kernel
// boundaries:
//   per layer: qkv GEMV (+RMSNorm, RoPE, KV append) | attention | o GEMV
//   (+residual) | gate/up GEMV (+RMSNorm, SwiGLU) | down GEMV (+residual)
//   then the lm_head GEMV with the greedy argmax.
// The producer warp of each CTA streams the CTA's share of EVERY weight of
// the step (all layers' tile-major chunks, then its lm_head rows) through
// the shared-memory ring without ever waiting for a barrier: weights do not
// depend on activations, so the next phase's weights are already arriving
// while the consumers wait at a barrier, build the activation operand and
// run attention (which reads the KV cache directly). The phase code is the
// standalone kernels' code (tiled_i8_consume, gemv_build_i8, attn_item).
//
// Data written in this launch by other CTAs (x, q, hidden) is read with L2
// loads (ld.global.cg): an SM's L1 is not kept coherent with other SMs'
// stores within a kernel.
//
// Grid barrier: counter bar[ph] per barrier of the step; each CTA adds 1
// after a __threadfence and spins (bounded by GEMV_WAIT_LIMIT_NS, and by the
// sticky error flag) until all CTAs have arrived. After passing barrier ph,
// CTA 0 clears bar[ph - 1] (every CTA has passed it), and bar[last] at the
// first barrier of the next step.
#pragma once

#include "attention.cuh"
#include "gemv_tiled.cuh"

#include <type_traits>

namespace aaedn_dev
{

struct LmMegaParams
{
    const float* hidden;
    const float* gain;
    const float* w; // [vocab][dim] fp32
    float* logits;
    float* part_val;
    int* part_idx;
    uint32_t* out_tokens;
    float eps;
    int dim, vocab, max_seq;
    int rows_per_cta;   // contiguous rows of one CTA
    int rows_per_chunk; // rows in one ring stage (1, 2, 4, 8 or 16)
};

struct MegaParams
{
    const GemvParams* gemv; // [n_layers][4]: qkv, o, gate/up, down
    const AttnParams* attn; // [n_layers]
    LmMegaParams lm;
    DecodeState* state;
    unsigned* bar; // [5 * n_layers] barrier counters, zero at the first launch
    int n_layers;
    int attn_items; // n_kv * S
    // tracing (null in normal runs): per CTA [MEGA_TRACE_CTA] cycle counts;
    // CTA 0's clock at the end of each phase's work and after each barrier
    unsigned long long* trace_cta;
    long long* trace_phase; // [5 * n_layers + 1][2]
};

// per-CTA trace slots
enum
{
    MT_CONS_WAIT = 0, // warp 0 of the consumers waiting for weight chunks
    MT_BARRIER,       // thread 0 in grid barriers
    MT_PROD_WAIT,     // the producer waiting for free stages
    MT_TOTAL,         // consumer thread 0, start to end
    MT_ATTN,          // attention phases (work only)
    MT_BUILD,         // activation builds
    MT_LM,            // lm_head phase
    MT_BUILD_A,       // activation builds: loads (pass A) only
    MEGA_TRACE_CTA = 8
};

// Shared memory: ring, barriers, then the work area (activation operand,
// attention groups or the lm_head input), the GEMV reduction buffers and
// scratch.
inline size_t mega_work_bytes(int max_ntile, size_t attn_bytes, int dim)
{
    size_t w = (size_t)max_ntile * (512 + 16); // operand tiles + block units
    const size_t a = 2 * ((attn_bytes + 15) / 16 * 16);
    if (a > w)
        w = a;
    const size_t l = (size_t)dim * 4 + 2 * 16 * 4;
    return w > l ? w : l;
}
inline size_t mega_smem_bytes(size_t work)
{
    return (size_t)GT_STAGES * GT_STAGE_BYTES + (size_t)GT_STAGES * 16 + work + GT_RED_BYTES + 64 * 4 +
           GT_ECACHE_FLOATS * 4;
}

// Consumer-side grid barrier (all NCT consumer threads of every CTA).
__device__ __forceinline__ bool mega_grid_sync(const MegaParams& P, int ph, int nph, volatile int& s_abort,
                                               unsigned long long* bar_cycles = nullptr)
{
    constexpr int NCT = GT_CONSUMERS * 32;
    named_bar_sync(1, NCT);
    bool failed = false;
    if (threadIdx.x == 0)
    {
        const long long c0 = clock64();
        if (P.trace_phase && blockIdx.x == 0)
            P.trace_phase[2 * ph] = c0;
        unsigned* ctr = P.bar + ph;
        __threadfence();
        asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(ctr) : "memory");
        const uint64_t t0 = globaltimer_ns();
        volatile uint32_t* err = &P.state->err;
        for (;;)
        {
            unsigned seen;
            asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(seen) : "l"(ctr) : "memory");
            if (seen >= gridDim.x)
                break;
            if (*err != 0u || globaltimer_ns() - t0 > GEMV_WAIT_LIMIT_NS)
            {
                P.state->err = 3u;
                s_abort = 1;
                failed = true;
                break;
            }
            __nanosleep(20);
        }
        __threadfence();
        if (blockIdx.x == 0 && !failed)
            P.bar[ph > 0 ? ph - 1 : nph - 1] = 0u;
        const long long c1 = clock64();
        if (bar_cycles)
            *bar_cycles += (unsigned long long)(c1 - c0);
        if (P.trace_phase && blockIdx.x == 0)
            P.trace_phase[2 * ph + 1] = c1;
    }
    return !named_bar_or(1, NCT, failed);
}

template <int G, int HDM>
__global__ void __launch_bounds__(GT_THREADS, 1) decode_step_kernel(const MegaParams P)
{
    constexpr int NS = GT_STAGES;
    constexpr int NC = GT_CONSUMERS;
    constexpr int NCT = NC * 32;
    extern __shared__ __align__(16) uint8_t smem[];
    __shared__ int s_abort_mem;
    __shared__ unsigned s_last[2];
    __shared__ float s_v[NC];
    __shared__ int s_i[NC];
    volatile int& s_abort = s_abort_mem;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int cta = blockIdx.x, ncta = gridDim.x;
    const int L = P.n_layers, nph = 5 * L;
    const LmMegaParams& lm = P.lm;

    // work area size: from the launch (dynamic smem size)
    uint32_t dyn_bytes;
    asm("mov.u32 %0, %%dynamic_smem_size;" : "=r"(dyn_bytes));
    const size_t work_bytes = dyn_bytes - ((size_t)NS * GT_STAGE_BYTES + (size_t)NS * 16 + GT_RED_BYTES + 64 * 4 +
                                           GT_ECACHE_FLOATS * 4);
    uint8_t* work = smem + (size_t)NS * GT_STAGE_BYTES + (size_t)NS * 16;
    float* red = reinterpret_cast<float*>(work + work_bytes);
    float* misc = red + GT_RED_BYTES / 4;
    float* ecache = misc + 64;
    TiledRing r;
    r.ring = smem_addr(smem);
    r.full = r.ring + NS * GT_STAGE_BYTES;
    r.empty = r.full + NS * 8;
    r.ns = NS;
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
        misc[48 + tid] = 0.0f; // 16 zero bytes: B operand of inactive lanes
    __syncthreads();

    // rows of the lm_head owned by this CTA
    const int n0 = cta * lm.rows_per_cta;
    const int nrows = max(0, min(lm.vocab, n0 + lm.rows_per_cta) - n0);
    const int R = lm.rows_per_chunk;
    const int nlchunk = (nrows + R - 1) / R;

    if (warp == NC)
    {
        // ---------------- producer warp: every weight of the step ----------------
        uint32_t q = 0;
        bool ok = true;
        unsigned long long pw = 0;
        unsigned long long* pwp = (P.trace_cta && lane == 0) ? &pw : nullptr;
        for (int l = 0; l < L && ok; ++l)
            for (int m = 0; m < 4 && ok; ++m)
            {
                const GemvParams& gp = P.gemv[4 * l + m];
                ok = tiled_produce(gp.w, gp.N, gp.K, r, q, cta, ncta, lane, pwp, gp.l2_hint != 0) && !s_abort;
            }
        for (int c = 0; c < nlchunk && ok; ++c, ++q)
        {
            const uint32_t stage = q % NS, use = q / NS;
            if (use > 0 && !mbar_wait_bounded(r.empty + 8 * stage, (use - 1) & 1, GEMV_WAIT_LIMIT_NS))
            {
                ok = false;
                break;
            }
            if (lane == 0)
            {
                const int rows = min(R, nrows - c * R);
                const uint32_t bytes = (uint32_t)rows * (uint32_t)lm.dim * 4u;
                mbar_arrive_expect_tx(r.full + 8 * stage, bytes);
                if (P.gemv[0].l2_hint)
                    bulk_g2s_hint(r.ring + stage * GT_STAGE_BYTES, lm.w + (size_t)(n0 + c * R) * lm.dim, bytes,
                                  r.full + 8 * stage, l2_evict_first_policy());
                else
                    bulk_g2s(r.ring + stage * GT_STAGE_BYTES, lm.w + (size_t)(n0 + c * R) * lm.dim, bytes,
                             r.full + 8 * stage);
            }
            __syncwarp();
        }
        if (!ok)
        {
            s_abort = 1;
            if (lane == 0)
                P.state->err = 2u;
        }
        tiled_drain(r, q);
        if (pwp)
            P.trace_cta[(size_t)cta * MEGA_TRACE_CTA + MT_PROD_WAIT] = pw;
        return;
    }

    // ---------------- consumer warps ----------------
    // trace accumulators in shared memory (thread 0 only, when tracing)
    __shared__ unsigned long long tr[MEGA_TRACE_CTA];
    const bool tracing = P.trace_cta != nullptr && tid == 0;
    if (tracing)
    {
        for (int k = 0; k < MEGA_TRACE_CTA; ++k)
            tr[k] = 0ull;
        tr[MT_TOTAL] = (unsigned long long)clock64();
    }
    unsigned long long* cw = tracing ? &tr[MT_CONS_WAIT] : nullptr;
    unsigned long long* bw = tracing ? &tr[MT_BARRIER] : nullptr;
    auto timed = [&](int slot, auto&& fn) {
        const long long c0 = tracing ? clock64() : 0;
        fn();
        if (tracing)
            tr[slot] += (unsigned long long)(clock64() - c0);
    };
    uint32_t q = 0;
    int ph = 0;
    bool ok = true;
    uint4* frag = reinterpret_cast<uint4*>(work);
    float* wss = misc + 32;
    const uint32_t zero16 = smem_addr(misc + 48);
    auto gemv = [&](auto pro, auto epi, const GemvParams& gp) -> bool {
        constexpr int PRO = decltype(pro)::value, EPI = decltype(epi)::value;
        float* bscale = reinterpret_cast<float*>(work + (size_t)(gp.K >> 7) * 512);
        timed(MT_BUILD, [&] { warp_build_i8<PRO>(gp, frag, bscale, wss, tracing ? &tr[MT_BUILD_A] : nullptr); });
        return tiled_wb_consume<PRO, EPI>(gp, r, q, frag, bscale, wss, zero16, red, ecache, cta, ncta, s_abort, cw);
    };
    using P_E = std::integral_constant<int, PRO_EMBED_RMSNORM>;
    using P_N = std::integral_constant<int, PRO_RMSNORM>;
    using P_P = std::integral_constant<int, PRO_PLAIN>;
    using P_A = std::integral_constant<int, PRO_ATTN_COMBINE>;
    using E_Q = std::integral_constant<int, EPI_QKV_ROPE>;
    using E_R = std::integral_constant<int, EPI_RESIDUAL>;
    using E_S = std::integral_constant<int, EPI_SWIGLU>;
    for (int l = 0; l < L && ok; ++l)
    {
        const GemvParams* gp = P.gemv + 4 * l;
        // qkv
        if (l > 0)
            ok = mega_grid_sync(P, ph++, nph, s_abort, bw);
        if (!ok)
            break;
        {
            // this CTA's attention rows of earlier positions (they do not
            // depend on this step) into L2 while the qkv phase runs
            const AttnParams& ap = P.attn[l];
            const int Lk = attn_len<1>(ap), lines = (ap.head_dim * 4 + 127) >> 7;
            for (int item = cta; item < P.attn_items; item += ncta)
            {
                int t0, t1;
                attn_range(Lk, item % ap.S, ap.S, t0, t1);
                const int pf1 = min(t1, min(Lk - 1, t0 + ATTN_PREFETCH_TOKENS));
                for (int i = tid; i < (pf1 - t0) * lines * 2; i += NCT)
                {
                    const int rr = i / (lines * 2), rem = i - rr * lines * 2, kv = rem / lines, ln = rem - kv * lines;
                    const size_t ro = attn_row<1>(ap, t0 + rr, item / ap.S);
                    asm volatile("prefetch.global.L2 [%0];" ::"l"((kv ? ap.v : ap.k) + ro + ln * 32));
                }
            }
        }
        ok = (l == 0 ? gemv(P_E{}, E_Q{}, gp[0]) : gemv(P_N{}, E_Q{}, gp[0])) &&
             mega_grid_sync(P, ph++, nph, s_abort, bw);
        if (!ok)
            break;
        // attention: two groups of 8 warps, items (kv head, split)
        timed(MT_ATTN, [&] {
            const AttnParams& ap = P.attn[l];
            const int wg = warp >> 3;
            float* asmem = reinterpret_cast<float*>(work) +
                           (size_t)wg * ((attn_smem_bytes(G, ap.head_dim, 0) + 15) / 16 * 4);
            for (int item = wg * ncta + cta; item < P.attn_items; item += 2 * ncta)
                attn_item<1, G, HDM>(ap, item / ap.S, item % ap.S, tid & 255, asmem, &s_last[wg], 2 + wg);
        });
        ok = mega_grid_sync(P, ph++, nph, s_abort, bw);
        if (!ok)
            break;
        // o (merges the attention splits as it builds its operand)
        ok = gemv(P_A{}, E_R{}, gp[1]) && mega_grid_sync(P, ph++, nph, s_abort, bw);
        if (!ok)
            break;
        // gate/up
        ok = gemv(P_N{}, E_S{}, gp[2]) && mega_grid_sync(P, ph++, nph, s_abort, bw);
        if (!ok)
            break;
        // down
        ok = gemv(P_P{}, E_R{}, gp[3]);
    }
    if (ok)
        ok = mega_grid_sync(P, ph++, nph, s_abort, bw);
    if (!ok)
    {
        if (lane == 0)
            P.state->err = P.state->err ? P.state->err : 2u;
        return;
    }
    if (tracing)
        tr[MT_LM] = (unsigned long long)clock64();

    // ---------------- lm_head: final RMSNorm, fp32 rows, argmax ----------------
    float* xs = reinterpret_cast<float*>(work);
    float* part = xs + lm.dim; // [2][16] partial dots, by chunk parity
    {
        float ss = 0.0f;
        // L2 loads (hidden was written by other CTAs in this launch)
        for (int i = tid; i < lm.dim; i += NCT)
        {
            const float h = __ldcg(lm.hidden + i);
            ss = fmaf(h, h, ss);
        }
        ss = group_sum<NCT>(ss, misc);
        const float rms = 1.0f / sqrtf(__fadd_rn(__fdiv_rn(ss, (float)lm.dim), lm.eps)); // src/transformer.cpp:230
        for (int i = tid; i < lm.dim; i += NCT)
            xs[i] = __fmul_rn(__fmul_rn(__ldcg(lm.hidden + i), rms), lm.gain[i]);
        named_bar_sync(1, NCT);
    }
    const int WPR = NC / R;              // warps per row
    const int slice4 = (lm.dim >> 2) / WPR; // float4 per warp slice
    const int row_in = warp / WPR, sl = warp - row_in * WPR;
    const uint32_t xs_a = smem_addr(xs);
    float bv = -INFINITY;
    int bi = INT_MAX;
    for (int c = 0; c < nlchunk; ++c, ++q)
    {
        const uint32_t stage = q % NS;
        if (!mbar_wait_bounded(r.full + 8 * stage, (q / NS) & 1, GEMV_WAIT_LIMIT_NS))
        {
            s_abort = 1;
            if (lane == 0)
                P.state->err = 2u;
            ok = false;
        }
        const int rows = min(R, nrows - c * R);
        float acc = 0.0f;
        if (ok && row_in < rows)
        {
            const uint32_t wr = r.ring + stage * GT_STAGE_BYTES + (uint32_t)row_in * (uint32_t)lm.dim * 4u;
            for (int k = sl * slice4 + lane; k < (sl + 1) * slice4; k += 32)
            {
                const uint4 wv = lds128(wr + (uint32_t)k * 16);
                const uint4 xv = lds128(xs_a + (uint32_t)k * 16);
                acc = fmaf(__uint_as_float(wv.x), __uint_as_float(xv.x), acc);
                acc = fmaf(__uint_as_float(wv.y), __uint_as_float(xv.y), acc);
                acc = fmaf(__uint_as_float(wv.z), __uint_as_float(xv.z), acc);
                acc = fmaf(__uint_as_float(wv.w), __uint_as_float(xv.w), acc);
            }
        }
        __syncwarp();
        if (lane == 0)
            mbar_arrive(r.empty + 8 * stage);
        acc = warp_sum(acc);
        float* pc = part + (c & 1) * NC;
        if (lane == 0)
            pc[warp] = acc;
        if (named_bar_or(1, NCT, !ok))
            break;
        if (tid < rows)
        {
            float v = 0.0f;
            for (int w = 0; w < WPR; ++w) // fixed order
                v += pc[tid * WPR + w];
            const int n = n0 + c * R + tid;
            lm.logits[n] = v;
            if (v > bv)
            {
                bv = v;
                bi = n;
            }
        }
    }
    if (tracing)
    {
        const unsigned long long t_end = (unsigned long long)clock64();
        tr[MT_LM] = t_end - tr[MT_LM];
        tr[MT_TOTAL] = t_end - tr[MT_TOTAL];
        for (int k = 0; k < MEGA_TRACE_CTA; ++k)
            if (k != MT_PROD_WAIT)
                P.trace_cta[(size_t)cta * MEGA_TRACE_CTA + k] = tr[k];
    }
    if (named_bar_or(1, NCT, !ok || s_abort))
        return; // decided together: every consumer returns
    // per-CTA best over the row owners (threads 0..R-1 of warp 0), then
    // across CTAs
    {
        float v = bv;
        int i = bi;
        if (warp == 0)
        {
#pragma unroll
            for (int o = 16; o > 0; o >>= 1)
            {
                const float ov = __shfl_xor_sync(0xffffffffu, v, o);
                const int oi = __shfl_xor_sync(0xffffffffu, i, o);
                if (ov > v || (ov == v && oi < i))
                {
                    v = ov;
                    i = oi;
                }
            }
            if (lane == 0)
            {
                lm.part_val[cta] = v;
                lm.part_idx[cta] = i;
                __threadfence();
                const unsigned prev = atomicAdd(&P.state->lm_counter, 1u);
                s_last[0] = prev == (unsigned)ncta - 1 ? 1u : 0u;
            }
        }
        named_bar_sync(1, NCT);
    }
    if (!s_last[0])
        return;
    __threadfence();
    float v = -INFINITY;
    int i = INT_MAX;
    for (int b = tid; b < ncta; b += NCT)
    {
        const float pv = __ldcg(lm.part_val + b);
        const int pi = __ldcg(lm.part_idx + b);
        if (pv > v || (pv == v && pi < i))
        {
            v = pv;
            i = pi;
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
    {
        const float ov = __shfl_xor_sync(0xffffffffu, v, o);
        const int oi = __shfl_xor_sync(0xffffffffu, i, o);
        if (ov > v || (ov == v && oi < i))
        {
            v = ov;
            i = oi;
        }
    }
    if (lane == 0)
    {
        s_v[warp] = v;
        s_i[warp] = i;
    }
    named_bar_sync(1, NCT);
    if (tid == 0)
    {
        v = s_v[0];
        i = s_i[0];
        for (int w = 1; w < NC; ++w)
            if (s_v[w] > v || (s_v[w] == v && s_i[w] < i))
            {
                v = s_v[w];
                i = s_i[w];
            }
        const uint32_t token = (i == INT_MAX) ? 0u : (uint32_t)i;
        DecodeState* st = P.state;
        const uint32_t pos = st->pos;
        if (pos + 1 >= st->n_prompt)
        {
            const uint32_t gi = pos + 1 - st->n_prompt;
            if (gi < (uint32_t)lm.max_seq)
                lm.out_tokens[gi] = token;
        }
        st->next_token = token;
        st->pos = pos + 1;
        st->lm_counter = 0u;
    }
}

} // namespace aaedn_dev
