// model.cu — the token loop on one B200: src/transformer.cpp:34-243
// (transformer_init / transformer_forward) rebuilt as a device-resident
// decode step.
//
// One step (one token at position pos) is 5 kernels per layer + 1:
//   qkv   : RMSNorm prologue (layer 0: embedding gather) -> fused QKV
//           dequant-GEMV -> RoPE on q,k -> k,v appended to the paged cache
//   attn  : split-K decode attention over the cache, GQA-aware
//   o     : dequant-GEMV + residual add into the hidden state
//   gu    : RMSNorm prologue -> fused gate/up dequant-GEMV -> silu(g)*u
//   down  : dequant-GEMV + residual add
//   lm    : final RMSNorm -> fp32 lm_head GEMV -> greedy argmax -> state
// The step reads its position and input token from device memory, so a
// whole step is captured once as a CUDA graph and replayed.
#include <algorithm>
#include <climits>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <vector>

#include "attention.cuh"
#include "gemm_tc.h"
#include "gemv_q4.cuh"
#include "gemv_tiled.cuh"
#include "prefill.cuh"
#include "tp.cuh"

namespace aaedn_dev
{
void repack_tiled(const uint8_t* codes, const uint16_t* scales, size_t N, size_t K, uint8_t* out)
{
    // the layout of gemv_tiled.cuh: per row group, chunks of <= 16 tiles;
    // tile codes [P][lane 4g + t][H0 r0, H0 r1, H1 r0, H1 r1] (4 bytes each:
    // bytes [8H + 4(t & 1), +4) of block 2P + (t >> 1) of row g + 8r), then
    // the chunk's tile scales [P][g][b'][r]
    const size_t ntile = K / 128, nchunk = (ntile + GT_CHUNK_TILES - 1) / GT_CHUNK_TILES;
    const size_t group_bytes = ntile * GT_TILE_BYTES;
    aaedn_host::parallel_for(N / 16, 1, [&](size_t g0, size_t g1) {
        for (size_t gi = g0; gi < g1; ++gi)
        {
            uint8_t* o = out + gi * group_bytes;
            for (size_t c = 0; c < nchunk; ++c)
            {
                const size_t tiles = std::min<size_t>(GT_CHUNK_TILES, ntile - c * GT_CHUNK_TILES);
                for (size_t i = 0; i < tiles; ++i)
                {
                    const size_t tile = c * GT_CHUNK_TILES + i;
                    for (int P = 0; P < 2; ++P)
                        for (int l = 0; l < 32; ++l)
                        {
                            const int g = l >> 2, t = l & 3;
                            const size_t blk = tile * 4 + 2 * P + (t >> 1);
                            for (int H = 0; H < 2; ++H)
                                for (int r = 0; r < 2; ++r)
                                {
                                    const size_t row = gi * 16 + g + 8 * r;
                                    std::memcpy(o, codes + row * (K / 2) + blk * 16 + 8 * H + 4 * (t & 1), 4);
                                    o += 4;
                                }
                        }
                }
                for (size_t i = 0; i < tiles; ++i)
                {
                    const size_t tile = c * GT_CHUNK_TILES + i;
                    for (int P = 0; P < 2; ++P)
                        for (int g = 0; g < 8; ++g)
                            for (int b = 0; b < 2; ++b)
                                for (int r = 0; r < 2; ++r)
                                {
                                    const size_t row = gi * 16 + g + 8 * r;
                                    std::memcpy(o, scales + row * (K / 32) + tile * 4 + 2 * P + b, 2);
                                    o += 2;
                                }
                }
            }
        }
    });
}
} // namespace aaedn_dev

using namespace aaedn_dev;

namespace
{

struct LmParams
{
    const float* hidden;
    const float* gain;
    float eps;
    int dim;
    const float* w; // [vocab][dim] fp32
    int vocab;
    float* logits;
    float* part_val;
    int* part_idx;
    DecodeState* state;
    uint32_t* out_tokens;
    int max_seq;
    int rows_per_cta;
    int stages;    // rows in the shared-memory ring, a multiple of consumers
    int consumers; // consumer warps that take rows (<= LM_CONSUMERS)
    int l2_hint;   // stream the rows with the L2 evict-first policy
    int row0;      // token id of row 0 (tensor parallel: this rank's first row)
    int defer;     // leave the per-CTA results (the ranks' argmax exchange finishes)
    unsigned long long* trace; // per-CTA timeline of a traced step, or null
};

constexpr int LM_CONSUMERS = 8;
constexpr int LM_THREADS = (LM_CONSUMERS + 1) * 32;
constexpr int LM_MAX_STAGES = 16;

// Shared memory of the lm_head kernel: the row ring, x, the barriers.
inline size_t lm_smem_bytes(int dim, int stages)
{
    return (size_t)stages * dim * 4 + (size_t)dim * 4 + (size_t)stages * 16 + 64 * 4;
}

// Final RMSNorm (src/transformer.cpp:230), fp32 lm_head GEMV
// (:232-238) and greedy argmax with ties to the lowest id; the last CTA
// advances the decode state.
//
// CTA b owns rows [b * rows_per_cta, ...): one contiguous run of the
// [vocab][dim] matrix. A producer warp streams it row by row with bulk copies
// into shared memory, starting before the programmatic-dependent wait (the
// weights do not depend on the previous kernel). Consumer warp w (w < C =
// p.consumers) takes rows w, w + C, ...; its k-th row lands in its own stage
// w + C * (k % SW) (SW = stages / C), so every stage is waited on by one warp,
// one use after the other (a parity wait two phases ahead would pass at once).
__global__ void __launch_bounds__(LM_THREADS, 1) lm_head_argmax_kernel(const LmParams p)
{
    constexpr int NC = LM_CONSUMERS;
    extern __shared__ __align__(16) uint8_t smem[];
    const int NS = p.stages, C = p.consumers, SW = NS / C;
    const uint32_t row_bytes = (uint32_t)p.dim * 4u;
    uint8_t* ring = smem;
    float* xs = reinterpret_cast<float*>(smem + (size_t)NS * row_bytes);
    uint64_t* bars = reinterpret_cast<uint64_t*>(xs + p.dim); // full[NS], empty[NS]
    float* misc = reinterpret_cast<float*>(bars + 2 * NS);
    __shared__ float s_v[NC];
    __shared__ int s_i[NC];
    __shared__ unsigned s_last;
    __shared__ int s_abort_mem;
    volatile int& s_abort = s_abort_mem;

    pdl_launch_dependents();
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (tid == 0)
        trace_mark(p.trace, blockIdx.x, 0);
    const int n0 = blockIdx.x * p.rows_per_cta;
    const int nrows = max(0, min(p.vocab, n0 + p.rows_per_cta) - n0);
    const uint32_t ring_a = smem_addr(ring);
    const uint32_t full_a = smem_addr(bars), empty_a = full_a + NS * 8;
    if (tid == 0)
    {
        for (int i = 0; i < NS; ++i)
        {
            mbar_init(full_a + 8 * i, 1);
            mbar_init(empty_a + 8 * i, 1);
        }
        mbar_init_fence();
        s_abort = 0;
    }
    __syncthreads();

    if (warp == NC)
    {
        // ---------------- producer warp ----------------
        bool ok = true;
        int j = 0;
        for (; j < nrows; ++j)
        {
            const int w = j % C, k = j / C;
            const uint32_t stage = (uint32_t)(w + C * (k % SW)), use = (uint32_t)(k / SW);
            if (use > 0 && !mbar_wait_bounded(empty_a + 8 * stage, (use - 1) & 1, GEMV_WAIT_LIMIT_NS))
            {
                ok = false;
                break;
            }
            if (lane == 0)
            {
                mbar_arrive_expect_tx(full_a + 8 * stage, row_bytes);
                if (p.l2_hint)
                    bulk_g2s_hint(ring_a + stage * row_bytes, p.w + (size_t)(n0 + j) * p.dim, row_bytes,
                                  full_a + 8 * stage, l2_evict_first_policy());
                else
                    bulk_g2s(ring_a + stage * row_bytes, p.w + (size_t)(n0 + j) * p.dim, row_bytes, full_a + 8 * stage);
            }
            __syncwarp();
        }
        if (!ok)
        {
            s_abort = 1;
            if (lane == 0)
                p.state->err = 2u;
        }
        // every issued copy has landed before the CTA may exit: the last
        // use of each stage that was issued
        for (int st = 0; st < NS; ++st)
        {
            const int w = st % C, slot = st / C;
            const int nk = j > w ? (j - w + C - 1) / C : 0; // rows issued to warp w
            if (nk > slot)
            {
                const int kl = slot + ((nk - 1 - slot) / SW) * SW; // last k with k % SW == slot
                mbar_wait_bounded(full_a + 8 * st, (uint32_t)(kl / SW) & 1, GEMV_WAIT_LIMIT_NS);
            }
        }
        return;
    }

    // ---------------- consumer warps ----------------
    pdl_wait(); // the hidden state comes from the previous kernel
    float ss = 0.0f;
    for (int i = tid; i < p.dim; i += NC * 32)
        ss = fmaf(p.hidden[i], p.hidden[i], ss);
    ss = group_sum<NC * 32>(ss, misc);
    const float rms = 1.0f / sqrtf(__fadd_rn(__fdiv_rn(ss, (float)p.dim), p.eps));
    for (int i = tid; i < p.dim; i += NC * 32)
        xs[i] = __fmul_rn(__fmul_rn(p.hidden[i], rms), p.gain[i]);
    named_bar_sync(1, NC * 32);
    if (tid == 0)
        trace_mark(p.trace, blockIdx.x, 1);

    const int d4 = p.dim >> 2;
    const uint32_t xs_a = smem_addr(xs);
    float bv = -INFINITY;
    int bi = INT_MAX;
    for (int j = warp, k = 0; warp < C && j < nrows; j += C, ++k)
    {
        const uint32_t stage = (uint32_t)(warp + C * (k % SW));
        if (!mbar_wait_bounded(full_a + 8 * stage, (uint32_t)(k / SW) & 1, GEMV_WAIT_LIMIT_NS) || s_abort)
        {
            s_abort = 1;
            if (lane == 0)
                p.state->err = 2u;
            break;
        }
        const uint32_t wr = ring_a + stage * row_bytes;
        float acc = 0.0f;
#pragma unroll 8
        for (int k = lane; k < d4; k += 32)
        {
            const uint4 wv = lds128(wr + (uint32_t)k * 16);
            const uint4 xv = lds128(xs_a + (uint32_t)k * 16);
            acc = fmaf(__uint_as_float(wv.x), __uint_as_float(xv.x), acc);
            acc = fmaf(__uint_as_float(wv.y), __uint_as_float(xv.y), acc);
            acc = fmaf(__uint_as_float(wv.z), __uint_as_float(xv.z), acc);
            acc = fmaf(__uint_as_float(wv.w), __uint_as_float(xv.w), acc);
        }
        __syncwarp();
        if (lane == 0)
            mbar_arrive(empty_a + 8 * stage);
        acc = warp_sum(acc);
        const int n = n0 + j;
        if (lane == 0)
            p.logits[n] = acc;
        if (acc > bv)
        {
            bv = acc;
            bi = n + p.row0;
        }
    }
    if (lane == 0)
    {
        s_v[warp] = bv;
        s_i[warp] = bi;
    }
    named_bar_sync(1, NC * 32);
    if (tid == 0)
    {
        float v = s_v[0];
        int i = s_i[0];
        for (int w = 1; w < NC; ++w)
            if (s_v[w] > v || (s_v[w] == v && s_i[w] < i))
            {
                v = s_v[w];
                i = s_i[w];
            }
        p.part_val[blockIdx.x] = v;
        p.part_idx[blockIdx.x] = i;
        trace_mark(p.trace, blockIdx.x, 3);
        s_last = 0u;
        if (!p.defer)
        {
            __threadfence();
            const unsigned prev = atomicAdd(&p.state->lm_counter, 1u);
            s_last = prev == gridDim.x - 1 ? 1u : 0u;
        }
    }
    named_bar_sync(1, NC * 32);
    if (!s_last)
        return;
    __threadfence();
    float v = -INFINITY;
    int i = INT_MAX;
    for (int b = tid; b < (int)gridDim.x; b += NC * 32)
    {
        const float pv = __ldcg(p.part_val + b);
        const int pi = __ldcg(p.part_idx + b);
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
    named_bar_sync(1, NC * 32);
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
        DecodeState* st = p.state;
        const uint32_t pos = st->pos;
        if (pos + 1 >= st->n_prompt)
        {
            const uint32_t gi = pos + 1 - st->n_prompt;
            if (gi < (uint32_t)p.max_seq)
                p.out_tokens[gi] = token;
        }
        st->next_token = token;
        st->pos = pos + 1;
        st->lm_counter = 0u;
    }
}

struct DevLayer
{
    // codes and scales of a matrix are one region: row-major codes followed
    // by the scales, or (when the shape tiles) the tile-major repacking
    uint8_t *wqkv, *wo, *wgu, *wd;
    uint16_t *sqkv, *so, *sgu, *sd;
    bool tqkv, to, tgu, td;
    float *attn_norm, *ffn_norm;
    float *k, *v; // [n_pages][n_kv][P][hd]
};

constexpr size_t TILED_SMEM_MAX = 226 * 1024; // under the 227 KB opt-in maximum of one CTA (static smem too)

inline bool tiles_ok(size_t N, size_t K)
{
    return N % 16 == 0 && K % 128 == 0 && K > 0 && gemv_tiled_i8_smem_bytes((int)(K / 128)) <= TILED_SMEM_MAX;
}

template <int PRO, int EPI>
int model_gemv(const GemvParams& p, cudaStream_t st, bool pdl, bool tiled = false)
{
    if (tiled)
    {
        static const int max_stages = [] {
            const char* e = std::getenv("AAEDN_GEMV_STAGES");
            return e ? std::max(GT_STAGES, std::min(GT_MAX_STAGES, std::atoi(e))) : 8;
        }();
        const int groups = p.N / 16;
        const int grid = groups < sm_count() ? groups : sm_count();
        GemvParams pp = p;
        pp.stages = std::min(max_stages, gemv_tiled_stages(p.K / 128, TILED_SMEM_MAX));
        cudaError_t e = launch_kernel(gemv_tiled_i8_kernel<PRO, EPI>, dim3(grid), dim3(GT_THREADS),
                                      gemv_tiled_i8_smem_bytes(p.K / 128, pp.stages), st, pdl, pp);
        if (e != cudaSuccess)
            return set_error(AAEDN_ECUDA, "launch of gemv_tiled_i8_kernel failed: %s", cudaGetErrorString(e));
        count_launch();
        return AAEDN_OK;
    }
    {
    auto kern = (p.full_shape && p.scale_pairs) ? gemv_q4_kernel<1, PRO, EPI, AAEDN_SCALE_F16, true>
                                                : gemv_q4_kernel<1, PRO, EPI, AAEDN_SCALE_F16, false>;
    static int per_sm = -1;
    if (per_sm < 0)
    {
        const char* e = std::getenv("AAEDN_GEMV_CTAS_PER_SM");
        per_sm = e ? std::max(1, std::atoi(e)) : 2;
    }
    const int groups = (p.N + 15) / 16;
    const int grid = groups < per_sm * sm_count() ? groups : per_sm * sm_count();
    const size_t smem = gemv_smem_bytes(1, p.kt1 - p.kt0);
    cudaError_t e = launch_kernel(kern, dim3(grid), dim3(GEMV_WARPS * 32), smem, st, pdl, p);
    if (e != cudaSuccess)
        return set_error(AAEDN_ECUDA, "launch of gemv_q4_kernel(model) failed: %s", cudaGetErrorString(e));
    count_launch();
    return AAEDN_OK;
    }
}

// Opt every model kernel into large dynamic shared memory once, before any
// stream capture.
template <int PRO, int EPI>
int set_gemv_attrs()
{
    AAEDN_CUDA_TRY(cudaFuncSetAttribute(gemv_q4_kernel<1, PRO, EPI, AAEDN_SCALE_F16, false>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
    AAEDN_CUDA_TRY(cudaFuncSetAttribute(gemv_q4_kernel<1, PRO, EPI, AAEDN_SCALE_F16, true>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
    AAEDN_CUDA_TRY(cudaFuncSetAttribute(gemv_tiled_i8_kernel<PRO, EPI>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, (int)TILED_SMEM_MAX));
    return AAEDN_OK;
}

int set_model_kernel_attrs()
{
    int rc = set_gemv_attrs<PRO_EMBED_RMSNORM, EPI_QKV_ROPE>();
    if (!rc)
        rc = set_gemv_attrs<PRO_RMSNORM, EPI_QKV_ROPE>();
    if (!rc)
        rc = set_gemv_attrs<PRO_PLAIN, EPI_RESIDUAL>();
    if (!rc)
        rc = set_gemv_attrs<PRO_RMSNORM, EPI_SWIGLU>();
    if (!rc)
        rc = set_gemv_attrs<PRO_PLAIN, EPI_TP_PUSH>();
    if (!rc && cudaFuncSetAttribute(attn_prefill_tiled_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    (int)attn_prefill_tiled_smem_bytes()) != cudaSuccess)
        rc = set_error(AAEDN_ECUDA, "attn_prefill_tiled_kernel smem attribute failed");
    if (!rc && (cudaFuncSetAttribute(lm_rows_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)lm_rows_smem_bytes()) != cudaSuccess ||
                cudaFuncSetAttribute(lm_rows_few_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     200 * 1024) != cudaSuccess))
        rc = set_error(AAEDN_ECUDA, "lm_rows kernel smem attributes failed");
    return rc;
}

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

} // namespace

struct aaedn_model
{
    aaedn_model_config cfg{};
    cudaStream_t stream = nullptr;
    uint8_t* arena = nullptr;
    size_t arena_bytes = 0, used = 0;
    std::vector<DevLayer> layers;
    float *embedding = nullptr, *final_norm = nullptr, *lm_head = nullptr;
    float *rope_cos = nullptr, *rope_sin = nullptr;
    DecodeState* state = nullptr;
    uint32_t *prompt = nullptr, *out_tokens = nullptr;
    int* page_table = nullptr;
    float *hidden = nullptr, *qbuf = nullptr, *attn_out = nullptr, *act = nullptr, *logits = nullptr;
    float* attn_part = nullptr;
    unsigned* attn_counters = nullptr;
    float* lm_part_val = nullptr;
    int* lm_part_idx = nullptr;
    float* dbg_hidden = nullptr;
    int page_size = 64, n_pages = 0;
    int attn_S = 1, attn_max_tok = 1;
    int attn_cS = 0; // splits of the clustered decode attention (0: splits merged through global memory)
    int attn_warps = ATTN_WARPS; // warps a CTA of the clustered decode attention (MHA, head_dim <= 128)
    int lm_ctas = 1, lm_rows = 8, lm_stages = 8, lm_consumers = 8;
    cudaGraphExec_t graph_exec = nullptr;
    uint32_t kernels_per_step = 0;
    uint32_t h_pos = 0;
    uint32_t* pinned = nullptr; // host staging: [max_seq] tokens + state words
    bool weights_set = false;
    bool pdl = true;   // programmatic dependent launch inside the decode graph
    bool tiled = true; // tile-major repacking of the matrices whose shape allows it
    bool l2_hint = true; // weight streams with the L2 evict-first policy
    // tensor parallelism: cfg holds this rank's dims (heads, ffn rows and
    // lm_head rows of the rank), full the model's
    aaedn_model_config full{};
    int tp_rank = 0, tp_size = 1;
    uint32_t v0 = 0;           // first lm_head row (token id) of this rank
    uint32_t kpo = 0, kpd = 0; // K of o and down (padded to whole tiles when sharded)
    uint8_t* tp_region = nullptr; // peer-visible: partials [2][dim], flags, argmax slots
    size_t tp_region_bytes = 0;
    void* tp_peer[TP_MAX] = {};
    TpComm tp{};
    bool tp_ready = false;
    unsigned* tp_epoch = nullptr;
    unsigned* tp_counter = nullptr; // last-CTA count of a partial-writing GEMV
    float* hidden2 = nullptr;       // residual ping-pong: qkv folds into hidden2, gate/up into hidden
    // prefill: chunks of up to pf_rows prompt tokens through the tensor-core
    // GEMM (0: the prompt runs as decode steps)
    int pf_rows = 0;
    float *pf_hidden = nullptr, *pf_q = nullptr, *pf_attn = nullptr, *pf_act = nullptr;
    void* pf_ws = nullptr;
    size_t pf_ws_bytes = 0;
    unsigned* pf_err = nullptr;
    // batched sequences (aaedn_model_create_batched): the KV pages are a pool
    // shared by up to max_seqs sequences, each with its own page table; a
    // page is held by every sequence that lists it (a fork shares the
    // parent's pages) and copied before a holder writes into it
    uint32_t max_seqs = 0; // 0: the single-sequence model
    uint32_t pt_stride = 0; // pages per sequence: its row of seq_pt
    int* seq_pt = nullptr;  // device [max_seqs][pt_stride]
    int *b_pos = nullptr, *b_seq = nullptr; // device [max_seqs]: the batch rows
    uint32_t *b_tokens = nullptr, *b_next = nullptr;
    float *b_logits = nullptr, *b_norm = nullptr; // [max_seqs][vocab], [max_seqs][dim]
    float* b_pval = nullptr;                     // greedy partials [max_seqs][b_parts]
    int* b_pidx = nullptr;
    int b_parts = 0;
    struct Seq
    {
        bool open = false;
        uint32_t len = 0;
        std::vector<int> pages;
    };
    std::vector<Seq> seqs;
    std::vector<int> page_ref, free_pages, h_pt;
    int* pinned_b = nullptr; // host staging: tokens, positions, sequences of a batch

    template <typename T>
    T* take(size_t bytes)
    {
        size_t off = align_up(used, 256);
        used = off + bytes;
        return reinterpret_cast<T*>(arena + off);
    }
};

static size_t plan_arena(aaedn_model* m, bool carve)
{
    const aaedn_model_config& c = m->cfg;
    const size_t D = c.dim, hd = c.head_dim, H = c.n_heads, KV = c.n_kv_heads, F = c.ffn_dim, V = c.vocab;
    const size_t qkv_rows = (H + 2 * KV) * hd;
    m->used = 0;
    if (carve)
        m->layers.resize(c.n_layers);
    for (uint32_t l = 0; l < c.n_layers; ++l)
    {
        DevLayer L{};
        auto mat = [&](uint8_t*& w, uint16_t*& sc, bool& tiled, size_t N, size_t K) {
            w = m->take<uint8_t>(N * K / 2 + N * K / 32 * 2);
            sc = reinterpret_cast<uint16_t*>(w + N * K / 2);
            tiled = m->tiled && tiles_ok(N, K);
        };
        mat(L.wqkv, L.sqkv, L.tqkv, qkv_rows, D);
        mat(L.wo, L.so, L.to, D, m->kpo);
        mat(L.wgu, L.sgu, L.tgu, 2 * F, D);
        mat(L.wd, L.sd, L.td, D, m->kpd);
        L.attn_norm = m->take<float>(D * 4);
        L.ffn_norm = m->take<float>(D * 4);
        L.k = m->take<float>((size_t)m->n_pages * KV * m->page_size * hd * 4);
        L.v = m->take<float>((size_t)m->n_pages * KV * m->page_size * hd * 4);
        if (carve)
            m->layers[l] = L;
    }
    m->embedding = m->take<float>((size_t)m->full.vocab * D * 4); // every rank: the whole table
    m->lm_head = m->take<float>(V * D * 4);
    m->final_norm = m->take<float>(D * 4);
    m->rope_cos = m->take<float>((size_t)c.max_seq * (hd / 2) * 4);
    m->rope_sin = m->take<float>((size_t)c.max_seq * (hd / 2) * 4);
    m->state = m->take<DecodeState>(sizeof(DecodeState));
    m->prompt = m->take<uint32_t>((size_t)c.max_seq * 4);
    m->out_tokens = m->take<uint32_t>((size_t)c.max_seq * 4);
    m->page_table = m->take<int>((size_t)m->n_pages * 4);
    m->hidden = m->take<float>(D * 4);
    m->qbuf = m->take<float>(H * hd * 4);
    m->attn_out = m->take<float>(std::max<size_t>(H * hd, m->kpo) * 4); // padding stays zero
    m->act = m->take<float>(std::max<size_t>(F, m->kpd) * 4);
    m->logits = m->take<float>(V * 4);
    m->attn_part = m->take<float>(H * (size_t)m->attn_S * (hd + 4) * 4);
    m->attn_counters = m->take<unsigned>(KV * 4);
    const size_t lm_parts = (size_t)std::max(m->lm_ctas, sm_count());
    m->lm_part_val = m->take<float>(lm_parts * 4);
    m->lm_part_idx = m->take<int>(lm_parts * 4);
    m->tp_epoch = m->take<unsigned>(64);
    m->tp_counter = m->take<unsigned>(64);
    m->hidden2 = m->take<float>(D * 4); // tensor parallel: the other residual buffer
    m->dbg_hidden = m->take<float>((size_t)c.n_layers * D * 4);
    if (m->pf_rows)
    {
        const size_t P = (size_t)m->pf_rows;
        m->pf_hidden = m->take<float>(P * D * 4);
        m->pf_q = m->take<float>(P * H * hd * 4);
        m->pf_attn = m->take<float>(P * m->kpo * 4);
        m->pf_act = m->take<float>(P * m->kpd * 4);
        size_t ws = 0;
        for (const auto& nk : {std::make_pair(qkv_rows, D), std::make_pair(D, (size_t)m->kpo),
                               std::make_pair(2 * F, D), std::make_pair(D, (size_t)m->kpd)})
            ws = std::max(ws, tc_gemm_workspace_bytes((int)P, (int)nk.first, (int)nk.second));
        m->pf_ws_bytes = ws;
        m->pf_ws = m->take<uint8_t>(ws);
        m->pf_err = m->take<unsigned>(64);
    }
    if (m->max_seqs)
    {
        const size_t S = m->max_seqs;
        m->seq_pt = m->take<int>(S * m->pt_stride * 4);
        m->b_pos = m->take<int>(S * 4);
        m->b_seq = m->take<int>(S * 4);
        m->b_tokens = m->take<uint32_t>(S * 4);
        m->b_next = m->take<uint32_t>(S * 4);
        m->b_logits = m->take<float>(S * V * 4);
        m->b_norm = m->take<float>(S * D * 4);
        m->b_parts = std::max((int)((V + LR_BN - 1) / LR_BN), 2 * sm_count());
        m->b_pval = m->take<float>(S * (size_t)m->b_parts * 4);
        m->b_pidx = m->take<int>(S * (size_t)m->b_parts * 4);
    }
    return align_up(m->used, 256);
}

// Kernel classes of a decode step (mask bits for the tracing sub-graphs).
enum
{
    K_QKV = 1,
    K_ATTN = 2,
    K_O = 4,
    K_GU = 8,
    K_DOWN = 16,
    K_LM = 32,
    K_ALL = 63,
};

// Parameters of the kernels of layer l (shared by the per-kernel decode
// graph and the persistent step kernel).
static GemvParams qkv_params(const aaedn_model* m, uint32_t l)
{
    const aaedn_model_config& c = m->cfg;
    const int D = (int)c.dim, hd = (int)c.head_dim, H = (int)c.n_heads, KV = (int)c.n_kv_heads;
    const DevLayer& L = m->layers[l];
    GemvParams q{};
    q.w = L.wqkv;
    q.s = L.sqkv;
    q.ldb = (size_t)D;
    q.N = (H + 2 * KV) * hd;
    q.K = D;
    q.kt0 = 0;
    q.kt1 = (D + 127) / 128;
    q.x = m->hidden;
    q.lda = (size_t)D;
    q.gain = L.attn_norm;
    q.eps = c.eps;
    q.embedding = m->embedding;
    q.prompt = m->prompt;
    q.state = m->state;
    q.hidden_out = m->hidden;
    q.q_rows = H * hd;
    q.kv_rows = KV * hd;
    q.head_dim = hd;
    q.n_kv = KV;
    q.page_size = m->page_size;
    q.max_pos = (int)c.max_seq;
    q.qbuf = m->qbuf;
    q.k_layer = L.k;
    q.v_layer = L.v;
    q.page_table = m->page_table;
    q.rope_cos = m->rope_cos;
    q.rope_sin = m->rope_sin;
    q.full_shape = (q.N % 16) == 0 && (q.K % 128) == 0;
    q.scale_pairs = ((D >> 5) & 1) == 0;
    q.l2_hint = m->l2_hint;
    return q;
}

static AttnParams attn_params(const aaedn_model* m, uint32_t l, int S)
{
    const aaedn_model_config& c = m->cfg;
    const int hd = (int)c.head_dim;
    const DevLayer& L = m->layers[l];
    AttnParams a{};
    a.q = m->qbuf;
    a.k = L.k;
    a.v = L.v;
    a.out = m->attn_out;
    a.part = m->attn_part;
    a.counters = m->attn_counters;
    a.n_heads = (int)c.n_heads;
    a.n_kv = (int)c.n_kv_heads;
    a.head_dim = hd;
    a.S = S;
    a.scale = 1.0f / std::sqrt((float)hd); // src/transformer.cpp:198
    a.state = m->state;
    a.max_len = (int)c.max_seq;
    a.max_tok = m->attn_max_tok;
    a.page_table = nullptr; // the sequence's pages are 0, 1, ... (identity table): no lookup before the K/V loads
    a.page_size = m->page_size;
    a.pstride = hd + 4; // 16-byte rows: the o-proj build reads them as float4
    a.warps = m->attn_warps;
    return a;
}

static GemvParams o_params(const aaedn_model* m, uint32_t l)
{
    const aaedn_model_config& c = m->cfg;
    const int D = (int)c.dim;
    const DevLayer& L = m->layers[l];
    GemvParams o{};
    o.w = L.wo;
    o.s = L.so;
    o.ldb = (size_t)m->kpo;
    o.N = D;
    o.K = (int)m->kpo;
    o.kt0 = 0;
    o.kt1 = ((int)m->kpo + 127) / 128;
    o.x = m->attn_out;
    o.lda = (size_t)m->kpo;
    o.y = m->hidden; // sharded: the rows are pushed to the ranks instead (EPI_TP_PUSH, buffer 0)
    o.ldc = (size_t)D;
    o.state = m->state;
    o.full_shape = (o.N % 16) == 0 && (o.K % 128) == 0;
    o.scale_pairs = ((m->kpo >> 5) & 1) == 0;
    o.l2_hint = m->l2_hint;
    if (m->tp_size > 1)
    {
        o.tpc = m->tp;
        o.tp_epoch = m->tp_epoch;
        o.tp_counter = m->tp_counter;
        o.tp_sig = 1;
        o.tp_sig_phase = 2 * (int)l;
        o.tp_buf = 0;
    }
    return o;
}

static GemvParams gu_params(const aaedn_model* m, uint32_t l)
{
    const aaedn_model_config& c = m->cfg;
    const int D = (int)c.dim, F = (int)c.ffn_dim;
    const DevLayer& L = m->layers[l];
    GemvParams gu{};
    gu.w = L.wgu;
    gu.s = L.sgu;
    gu.ldb = (size_t)D;
    gu.N = 2 * F;
    gu.K = D;
    gu.kt0 = 0;
    gu.kt1 = (D + 127) / 128;
    gu.x = m->hidden;
    gu.lda = (size_t)D;
    gu.gain = L.ffn_norm;
    gu.eps = c.eps;
    gu.act = m->act;
    gu.state = m->state;
    gu.full_shape = (gu.N % 16) == 0 && (gu.K % 128) == 0;
    gu.scale_pairs = ((D >> 5) & 1) == 0;
    gu.l2_hint = m->l2_hint;
    return gu;
}

static GemvParams down_params(const aaedn_model* m, uint32_t l)
{
    const aaedn_model_config& c = m->cfg;
    const int D = (int)c.dim;
    const DevLayer& L = m->layers[l];
    GemvParams dn{};
    dn.w = L.wd;
    dn.s = L.sd;
    dn.ldb = (size_t)m->kpd;
    dn.N = D;
    dn.K = (int)m->kpd;
    dn.kt0 = 0;
    dn.kt1 = ((int)m->kpd + 127) / 128;
    dn.x = m->act;
    dn.lda = (size_t)m->kpd;
    dn.y = m->hidden; // sharded: pushed to the ranks (EPI_TP_PUSH, buffer 1)
    dn.ldc = (size_t)D;
    dn.state = m->state;
    dn.full_shape = (dn.N % 16) == 0 && (dn.K % 128) == 0;
    dn.scale_pairs = ((m->kpd >> 5) & 1) == 0;
    dn.l2_hint = m->l2_hint;
    if (m->tp_size > 1)
    {
        dn.tpc = m->tp;
        dn.tp_epoch = m->tp_epoch;
        dn.tp_counter = m->tp_counter;
        dn.tp_sig = 1;
        dn.tp_sig_phase = 2 * (int)l + 1;
        dn.tp_buf = 1;
    }
    return dn;
}

static LmParams lm_params(const aaedn_model* m)
{
    const aaedn_model_config& c = m->cfg;
    LmParams lp{};
    lp.hidden = m->hidden;
    lp.gain = m->final_norm;
    lp.eps = c.eps;
    lp.dim = (int)c.dim;
    lp.w = m->lm_head;
    lp.vocab = (int)c.vocab;
    lp.logits = m->logits;
    lp.part_val = m->lm_part_val;
    lp.part_idx = m->lm_part_idx;
    lp.state = m->state;
    lp.out_tokens = m->out_tokens;
    lp.max_seq = (int)c.max_seq;
    lp.rows_per_cta = m->lm_rows;
    lp.stages = m->lm_stages;
    lp.consumers = m->lm_consumers;
    lp.l2_hint = m->l2_hint;
    lp.row0 = (int)m->v0;
    lp.defer = m->tp_size > 1 ? 1 : 0;
    return lp;
}

// hidden += the sum of the ranks' partials in buffer buf (o: 0, down: 1)
static int tp_reduce(aaedn_model* m, cudaStream_t st, int buf, int phase, bool signal, bool pdl)
{
    if (!m->tp_ready)
        return set_error(AAEDN_ESTATE, "tensor parallel model: aaedn_model_tp_connect was not called");
    TpReduceParams rp{};
    rp.c = m->tp;
    rp.hidden = m->hidden;
    rp.dim = (int)m->cfg.dim;
    rp.buf = buf;
    rp.phase = phase;
    rp.signal = signal ? 1 : 0;
    rp.epoch = m->tp_epoch;
    rp.state = m->state;
    const int blocks = std::max(1, std::min(32, (int)(m->cfg.dim + 255) / 256));
    cudaError_t e = launch_kernel(tp_reduce_kernel, dim3(blocks), dim3(256), 0, st, pdl, rp);
    if (e != cudaSuccess)
        return set_error(AAEDN_ECUDA, "launch of tp_reduce_kernel failed: %s", cudaGetErrorString(e));
    count_launch();
    return AAEDN_OK;
}

// trace: a timeline buffer of [5 n_layers + 1][STEP_TRACE_CTAS][STEP_TRACE_EVENTS]
// stamps (qkv, attention, o, gate/up, down of each layer, then lm_head), or null
static int enqueue_step(aaedn_model* m, cudaStream_t st, bool debug, const std::vector<cudaEvent_t>* ev = nullptr,
                        int mask = K_ALL, unsigned long long* trace = nullptr)
{
    if (m->tp_size > 1 && !m->tp_ready)
        return set_error(AAEDN_ESTATE, "tensor parallel model: aaedn_model_tp_connect was not called");
    // programmatic dependent launches between consecutive kernels (not when
    // events or copies sit between them)
    const bool pdl = m->pdl && !ev && !debug;
    size_t evi = 0;
    auto mark = [&]() -> int {
        // external event nodes: timestamps are taken inside the graph
        if (ev && evi < ev->size())
            AAEDN_CUDA_TRY(cudaEventRecordWithFlags((*ev)[evi++], st, cudaEventRecordExternal));
        return AAEDN_OK;
    };
    int mrc = mark();
    if (mrc)
        return mrc;
    const aaedn_model_config& c = m->cfg;
    const int D = (int)c.dim, KV = (int)c.n_kv_heads;
    int rc;
    for (uint32_t l = 0; l < c.n_layers; ++l)
    {
        const DevLayer& L = m->layers[l];
        GemvParams q = qkv_params(m, l), o = o_params(m, l), gu = gu_params(m, l), dn = down_params(m, l);
        const int aS = m->attn_cS ? m->attn_cS : m->attn_S;
        AttnParams a = attn_params(m, l, aS);
        if (trace)
        {
            const size_t per = (size_t)STEP_TRACE_CTAS * STEP_TRACE_EVENTS, k0 = (size_t)l * 5;
            q.trace = trace + k0 * per;
            a.trace = trace + (k0 + 1) * per;
            o.trace = trace + (k0 + 2) * per;
            gu.trace = trace + (k0 + 3) * per;
            dn.trace = trace + (k0 + 4) * per;
        }
        // --- QKV (+RMSNorm prologue, +RoPE/KV-append epilogue)
        rc = !(mask & K_QKV) ? AAEDN_OK
             : (l == 0)      ? model_gemv<PRO_EMBED_RMSNORM, EPI_QKV_ROPE>(q, st, pdl, L.tqkv)
                             : model_gemv<PRO_RMSNORM, EPI_QKV_ROPE>(q, st, pdl, L.tqkv);
        if (rc)
            return rc;
        if ((rc = mark()))
            return rc;
        // --- attention
        rc = !(mask & K_ATTN) ? AAEDN_OK
             : m->attn_cS     ? attn_launch_cluster(a, dim3(KV, aS), st, pdl)
                              : attn_launch_global(a, dim3(KV, aS), st, pdl);
        if (rc)
            return rc;
        if ((rc = mark()))
            return rc;
        // --- O projection + residual (sharded: this rank's partial, then the
        // reduction over the ranks adds the sum to the residual)
        if (m->tp_size > 1) // its partial, then the ranks' sum into the residual
        {
            rc = !(mask & K_O) ? AAEDN_OK : model_gemv<PRO_PLAIN, EPI_TP_PUSH>(o, st, pdl, L.to);
            if (!rc && (mask & K_O))
                rc = tp_reduce(m, st, 0, 2 * (int)l, false, pdl);
        }
        else
            rc = !(mask & K_O) ? AAEDN_OK : model_gemv<PRO_PLAIN, EPI_RESIDUAL>(o, st, pdl, L.to);
        if (rc)
            return rc;
        if ((rc = mark()))
            return rc;
        // --- gate/up (+RMSNorm prologue, SwiGLU epilogue)
        rc = !(mask & K_GU) ? AAEDN_OK : model_gemv<PRO_RMSNORM, EPI_SWIGLU>(gu, st, pdl, L.tgu);
        if (rc)
            return rc;
        if ((rc = mark()))
            return rc;
        // --- down + residual
        if (m->tp_size > 1) // its partial, then the ranks' sum into the residual
        {
            rc = (mask & K_DOWN) ? model_gemv<PRO_PLAIN, EPI_TP_PUSH>(dn, st, pdl, L.td) : AAEDN_OK;
            if (!rc && (mask & K_DOWN))
                rc = tp_reduce(m, st, 1, 2 * (int)l + 1, false, pdl);
        }
        else
            rc = (mask & K_DOWN) ? model_gemv<PRO_PLAIN, EPI_RESIDUAL>(dn, st, pdl, L.td) : AAEDN_OK;
        if (rc)
            return rc;
        if ((rc = mark()))
            return rc;
        if (debug)
            AAEDN_CUDA_TRY(cudaMemcpyAsync(m->dbg_hidden + (size_t)l * D, m->hidden, (size_t)D * 4,
                                           cudaMemcpyDeviceToDevice, st));
    }
    LmParams lp = lm_params(m);
    if (trace)
        lp.trace = trace + (size_t)c.n_layers * 5 * STEP_TRACE_CTAS * STEP_TRACE_EVENTS;
    if (mask & K_LM)
    {
        cudaError_t e = launch_kernel(lm_head_argmax_kernel, dim3(m->lm_ctas), dim3(LM_THREADS),
                                      lm_smem_bytes(D, m->lm_stages), st, pdl, lp);
        if (e != cudaSuccess)
            return set_error(AAEDN_ECUDA, "launch of lm_head_argmax_kernel failed: %s", cudaGetErrorString(e));
        count_launch();
        if (m->tp_size > 1)
        {
            TpArgmaxParams ap{};
            ap.c = m->tp;
            ap.part_val = m->lm_part_val;
            ap.part_idx = m->lm_part_idx;
            ap.n_parts = m->lm_ctas;
            ap.phase = 2 * (int)c.n_layers;
            ap.epoch = m->tp_epoch;
            ap.state = m->state;
            ap.out_tokens = m->out_tokens;
            ap.max_seq = (int)c.max_seq;
            cudaError_t ea = launch_kernel(tp_argmax_kernel, dim3(1), dim3(256), 0, st, pdl, ap);
            if (ea != cudaSuccess)
                return set_error(AAEDN_ECUDA, "launch of tp_argmax_kernel failed: %s", cudaGetErrorString(ea));
            count_launch();
        }
    }
    if (m->tp_size > 1)
    {
        // one step's worth of epochs, whatever part of the step was enqueued
        tp_epoch_kernel<<<1, 32, 0, st>>>(m->tp_epoch, 2u * c.n_layers + 1u);
        AAEDN_LAUNCH_CHECK("tp_epoch_kernel");
    }
    if ((rc = mark()))
        return rc;
    return AAEDN_OK;
}

static int ensure_graph(aaedn_model* m)
{
    if (m->graph_exec)
        return AAEDN_OK;
    const uint64_t before = g_launches.load();
    AAEDN_CUDA_TRY(cudaStreamBeginCapture(m->stream, cudaStreamCaptureModeThreadLocal));
    int rc = enqueue_step(m, m->stream, false);
    cudaGraph_t g = nullptr;
    cudaError_t e = cudaStreamEndCapture(m->stream, &g);
    const uint64_t after = g_launches.load();
    g_launches.fetch_sub(after - before);
    m->kernels_per_step = (uint32_t)(after - before);
    if (rc)
    {
        if (g)
            cudaGraphDestroy(g);
        return rc;
    }
    if (e != cudaSuccess)
        return set_error(AAEDN_ECUDA, "graph capture failed: %s", cudaGetErrorString(e));
    e = cudaGraphInstantiate(&m->graph_exec, g, 0);
    cudaGraphDestroy(g);
    if (e != cudaSuccess)
    {
        m->graph_exec = nullptr;
        return set_error(AAEDN_ECUDA, "graph instantiate failed: %s", cudaGetErrorString(e));
    }
    return AAEDN_OK;
}

static int run_steps(aaedn_model* m, size_t n)
{
    int rc = ensure_graph(m);
    if (rc)
        return rc;
    for (size_t i = 0; i < n; ++i)
    {
        AAEDN_CUDA_TRY(cudaGraphLaunch(m->graph_exec, m->stream));
        count_launch(m->kernels_per_step);
    }
    return AAEDN_OK;
}

// pos / n_prompt words of the device state
static int write_state(aaedn_model* m, uint32_t pos, uint32_t n_prompt)
{
    uint32_t* st = m->pinned + m->cfg.max_seq;
    st[0] = pos;
    st[1] = n_prompt;
    AAEDN_CUDA_TRY(cudaMemcpyAsync(m->state, st, 8, cudaMemcpyHostToDevice, m->stream));
    return AAEDN_OK;
}

// Synchronises and reports the device-side error flag of the decode state:
// 1 = a position past the cache, 2 = a weight-stream wait ran out, 3 = a
// grid barrier of the persistent kernel ran out, 4 = a wait for another
// tensor-parallel rank ran out. The flag stays set until aaedn_model_reset.
static int device_status(aaedn_model* m)
{
    uint32_t* w = m->pinned + m->cfg.max_seq + 4;
    AAEDN_CUDA_TRY(cudaMemcpyAsync(w, &m->state->err, 4, cudaMemcpyDeviceToHost, m->stream));
    if (m->pf_err)
        AAEDN_CUDA_TRY(cudaMemcpyAsync(w + 1, m->pf_err, 4, cudaMemcpyDeviceToHost, m->stream));
    AAEDN_CUDA_TRY(cudaStreamSynchronize(m->stream));
    if (m->pf_err && w[1] != 0u && *w == 0u)
        return set_error(AAEDN_ETIMEOUT, "a bounded wait of a prefill GEMM ran out");
    switch (*w)
    {
    case 0: return AAEDN_OK;
    case 1: return set_error(AAEDN_ESTATE, "decode step past the cache capacity (max_seq %u)", m->cfg.max_seq);
    case 4: return set_error(AAEDN_ETIMEOUT, "a wait for another tensor-parallel rank ran out");
    default: return set_error(AAEDN_ETIMEOUT, "a bounded device wait ran out (code %u)", *w);
    }
}

static int put_tokens(aaedn_model* m, const uint32_t* h_tokens, size_t n)
{
    // staging must not be rewritten while an earlier copy may still read it
    AAEDN_CUDA_TRY(cudaStreamSynchronize(m->stream));
    std::memcpy(m->pinned, h_tokens, n * 4);
    AAEDN_CUDA_TRY(cudaMemcpyAsync(m->prompt + m->h_pos, m->pinned, n * 4, cudaMemcpyHostToDevice, m->stream));
    return AAEDN_OK;
}

// Where the rows of a layer pass sit: row t at position pos0 + t of the one
// sequence whose page table is page_table (a prefill chunk), or, with
// row_pos / row_seq, at position row_pos[t] of sequence row_seq[t] whose page
// table starts at page_table + row_seq[t] * pt_stride (batched decode).
struct RowMap
{
    const int* page_table;
    uint32_t pos0;
    const int* row_pos;
    const int* row_seq;
    int pt_stride;
};

// The transformer layers over n residual rows in m->pf_hidden (the token
// loop of src/transformer.cpp:148-228 for many tokens at once): per layer
// RMSNorm -> QKV GEMM (RoPE, K/V appended to each row's page) -> causal
// attention -> O GEMM (+residual) -> RMSNorm -> gate/up GEMM (SwiGLU) ->
// down GEMM (+residual).
static int layers_pass(aaedn_model* m, int n, const RowMap& rm)
{
    cudaStream_t st = m->stream;
    const aaedn_model_config& c = m->cfg;
    const int D = (int)c.dim, H = (int)c.n_heads, KV = (int)c.n_kv_heads, hd = (int)c.head_dim, F = (int)c.ffn_dim;
    const int M_pad = tc_m_pad(n);
    __nv_bfloat16* parts = static_cast<__nv_bfloat16*>(tc_gemm_parts(m->pf_ws));
    TcGemmArgs base{};
    base.x = nullptr; // parts written into the workspace by the kernel before
    base.M = n;
    base.w_layout = TC_W_TILED;
    base.workspace = m->pf_ws;
    base.workspace_bytes = m->pf_ws_bytes;
    base.err = m->pf_err;
    int rc;
    for (uint32_t l = 0; l < c.n_layers; ++l)
    {
        const DevLayer& L = m->layers[l];
        // ---- attention block
        pf_rmsnorm_split_kernel<<<M_pad, 256, 0, st>>>(m->pf_hidden, D, n, M_pad, L.attn_norm, c.eps, parts);
        AAEDN_LAUNCH_CHECK("pf_rmsnorm_split_kernel");
        TcGemmArgs q = base;
        q.N = (H + 2 * KV) * hd;
        q.K = D;
        q.w = L.wqkv;
        q.epi = TC_EPI_QKV;
        q.e.qrows = m->pf_q;
        q.e.ldq = (size_t)H * hd;
        q.e.k_layer = L.k;
        q.e.v_layer = L.v;
        q.e.page_table = rm.page_table;
        q.e.page_size = m->page_size;
        q.e.n_kv = KV;
        q.e.head_dim = hd;
        q.e.q_rows = H * hd;
        q.e.kv_rows = KV * hd;
        q.e.pos0 = (int)rm.pos0;
        q.e.row_pos = rm.row_pos;
        q.e.row_seq = rm.row_seq;
        q.e.pt_stride = rm.pt_stride;
        q.e.rope_cos = m->rope_cos;
        q.e.rope_sin = m->rope_sin;
        if ((rc = tc_gemm(q, st)))
            return rc;
        if (rm.row_pos)
        {
            // batched decode: one query row per sequence, the decode kernel
            // with a cluster of S splits per (kv head, row), S making about
            // two CTAs per SM (a power of two, at most 8)
            int S = std::max(1, std::min(8, 2 * sm_count() / std::max(1, KV * n)));
            while (S & (S - 1))
                S &= S - 1;
            AttnParams a{};
            a.q = m->pf_q;
            a.ldq = (size_t)H * hd;
            a.k = L.k;
            a.v = L.v;
            a.out = m->pf_attn;
            a.ldo = m->kpo;
            a.n_heads = H;
            a.n_kv = KV;
            a.head_dim = hd;
            a.S = S;
            a.scale = 1.0f / std::sqrt((float)hd); // src/transformer.cpp:198
            a.max_len = (int)c.max_seq;
            a.page_table = rm.page_table;
            a.page_size = m->page_size;
            a.row_pos = rm.row_pos;
            a.row_seq = rm.row_seq;
            a.pt_stride = rm.pt_stride;
            if ((rc = attn_launch_cluster(a, dim3(KV, S, n), st, false)))
                return rc;
        }
        else if (hd <= 128 && hd % 4 == 0 && m->page_size % PFT_K == 0)
        {
            attn_prefill_tiled_kernel<<<dim3(H, (n + PFT_Q - 1) / PFT_Q), PFT_WARPS * 32,
                                        attn_prefill_tiled_smem_bytes(), st>>>(
                m->pf_q, (size_t)H * hd, L.k, L.v, rm.page_table, m->page_size, H, KV, hd, (int)rm.pos0, n,
                1.0f / std::sqrt((float)hd), m->pf_attn, m->kpo);
            AAEDN_LAUNCH_CHECK("attn_prefill_tiled_kernel");
        }
        else
        {
            attn_prefill_kernel<<<dim3(H, (n + PF_ATTN_WARPS - 1) / PF_ATTN_WARPS), PF_ATTN_WARPS * 32, 0, st>>>(
                m->pf_q, (size_t)H * hd, L.k, L.v, rm.page_table, m->page_size, H, KV, hd, (int)rm.pos0, n,
                1.0f / std::sqrt((float)hd), m->pf_attn, m->kpo);
            AAEDN_LAUNCH_CHECK("attn_prefill_kernel");
        }
        if ((rc = tc_split(m->pf_attn, m->kpo, n, (int)m->kpo, m->pf_ws, st)))
            return rc;
        TcGemmArgs o = base;
        o.N = D;
        o.K = (int)m->kpo;
        o.w = L.wo;
        o.epi = TC_EPI_RESID;
        o.out = m->pf_hidden;
        o.ldc = (size_t)D;
        if ((rc = tc_gemm(o, st)))
            return rc;
        // ---- feed-forward block
        pf_rmsnorm_split_kernel<<<M_pad, 256, 0, st>>>(m->pf_hidden, D, n, M_pad, L.ffn_norm, c.eps, parts);
        AAEDN_LAUNCH_CHECK("pf_rmsnorm_split_kernel");
        TcGemmArgs gu = base;
        gu.N = 2 * F;
        gu.K = D;
        gu.w = L.wgu;
        gu.epi = TC_EPI_SWIGLU;
        gu.e.act = m->pf_act;
        gu.e.ld_act = m->kpd;
        if ((rc = tc_gemm(gu, st)))
            return rc;
        if ((rc = tc_split(m->pf_act, m->kpd, n, (int)m->kpd, m->pf_ws, st)))
            return rc;
        TcGemmArgs dn = base;
        dn.N = D;
        dn.K = (int)m->kpd;
        dn.w = L.wd;
        dn.epi = TC_EPI_RESID;
        dn.out = m->pf_hidden;
        dn.ldc = (size_t)D;
        if ((rc = tc_gemm(dn, st)))
            return rc;
    }
    return AAEDN_OK;
}

// One chunk of n prompt tokens (d_tokens, device) of one sequence at
// positions pos0..: their residual rows (src/transformer.cpp:144-146), then
// the layers.
static int prefill_chunk(aaedn_model* m, const uint32_t* d_tokens, int n, const RowMap& rm)
{
    pf_embed_kernel<<<n, 256, 0, m->stream>>>(d_tokens, n, m->embedding, (int)m->cfg.dim, m->pf_hidden);
    AAEDN_LAUNCH_CHECK("pf_embed_kernel");
    return layers_pass(m, n, rm);
}

// n prompt tokens (already in m->prompt at h_pos) through prefill chunks,
// then the lm_head step of the last one: the decode state ends as after n
// decode steps (position h_pos + n, the greedy token of the last logits).
static int prefill(aaedn_model* m, size_t n)
{
    const uint32_t p0 = m->h_pos;
    int rc = AAEDN_OK;
    size_t last = 0;
    for (size_t c0 = 0; c0 < n && !rc; c0 += (size_t)m->pf_rows)
    {
        const int nc = (int)std::min<size_t>((size_t)m->pf_rows, n - c0);
        rc = prefill_chunk(m, m->prompt + p0 + c0, nc, RowMap{m->page_table, p0 + (uint32_t)c0, nullptr, nullptr, 0});
        last = (size_t)nc - 1;
    }
    if (rc)
        return rc;
    AAEDN_CUDA_TRY(cudaMemcpyAsync(m->hidden, m->pf_hidden + last * m->cfg.dim, (size_t)m->cfg.dim * 4,
                                   cudaMemcpyDeviceToDevice, m->stream));
    // the lm_head of the last prompt token as the decode step does it
    if ((rc = write_state(m, p0 + (uint32_t)n - 1, p0 + (uint32_t)n)))
        return rc;
    LmParams lp = lm_params(m);
    cudaError_t e = launch_kernel(lm_head_argmax_kernel, dim3(m->lm_ctas), dim3(LM_THREADS),
                                  lm_smem_bytes((int)m->cfg.dim, m->lm_stages), m->stream, false, lp);
    if (e != cudaSuccess)
        return set_error(AAEDN_ECUDA, "launch of lm_head_argmax_kernel failed: %s", cudaGetErrorString(e));
    count_launch();
    return AAEDN_OK;
}

#define MODEL_OK(m)                                                                                           \
    do                                                                                                        \
    {                                                                                                         \
        if (!(m))                                                                                             \
            return set_error(AAEDN_EINVAL, "null model");                                                    \
    } while (0)

extern "C" int aaedn_tp_plan_get(const aaedn_model_config* cfg, uint32_t tp_rank, uint32_t tp_size,
                                 aaedn_tp_plan* out)
{
    if (!cfg || !out)
        return set_error(AAEDN_EINVAL, "aaedn_tp_plan_get: null argument");
    const aaedn_model_config& fc = *cfg;
    if (tp_size != 1 && tp_size != 2 && tp_size != 4 && tp_size != 8)
        return set_error(AAEDN_EINVAL, "tensor parallel size must be 1, 2, 4 or 8");
    if (tp_rank >= tp_size || fc.n_kv_heads == 0 || fc.n_kv_heads % tp_size || fc.n_heads % tp_size ||
        fc.ffn_dim % (32 * tp_size) || fc.vocab < tp_size || (tp_size > 1 && fc.dim % 128))
        return set_error(AAEDN_EINVAL,
                         "rank %u of %u: n_heads, n_kv_heads and ffn_dim / 32 must divide by the tensor-parallel "
                         "size (and dim be a multiple of 128)",
                         tp_rank, tp_size);
    aaedn_tp_plan p{};
    p.n_heads = fc.n_heads / tp_size;
    p.n_kv_heads = fc.n_kv_heads / tp_size;
    p.ffn_dim = fc.ffn_dim / tp_size;
    const uint32_t vper = (fc.vocab + tp_size - 1) / tp_size;
    p.vocab0 = tp_rank * vper;
    p.vocab = p.vocab0 < fc.vocab ? std::min(vper, fc.vocab - p.vocab0) : 0u;
    p.q_head0 = tp_rank * p.n_heads;
    p.kv_head0 = tp_rank * p.n_kv_heads;
    p.ffn_row0 = tp_rank * p.ffn_dim;
    const uint32_t ko = p.n_heads * fc.head_dim, kd = p.ffn_dim;
    // sharded K of o and down: padded to whole 128-column tiles (zero
    // weights, zero activations) so the tile-major GEMV serves them
    p.o_k = tp_size > 1 ? (ko + 127) / 128 * 128 : ko;
    p.down_k = tp_size > 1 ? (kd + 127) / 128 * 128 : kd;
    if (p.vocab == 0 || (p.n_heads * fc.head_dim) % 32)
        return set_error(AAEDN_EINVAL, "rank %u of %u: no share left", tp_rank, tp_size);
    *out = p;
    return AAEDN_OK;
}

static int create_impl(const aaedn_model_config* cfg, uint32_t tp_rank, uint32_t tp_size, aaedn_model** out,
                       uint32_t max_seqs = 0, uint64_t kv_tokens = 0)
{
    if (!cfg || !out)
        return set_error(AAEDN_EINVAL, "aaedn_model_create: null argument");
    *out = nullptr;
    const aaedn_model_config& fc = *cfg;
    if (fc.dim == 0 || fc.n_layers == 0 || fc.n_heads == 0 || fc.n_kv_heads == 0 || fc.head_dim == 0 || fc.ffn_dim == 0 ||
        fc.vocab == 0 || fc.max_seq == 0)
        return set_error(AAEDN_EINVAL, "aaedn_model_create: zero dimension");
    if (fc.dim % 32 || (fc.n_heads * fc.head_dim) % 32 || fc.ffn_dim % 32 || fc.head_dim % 16 || fc.dim % 4 ||
        fc.n_heads % fc.n_kv_heads || fc.head_dim > (uint32_t)ATTN_MAX_HD ||
        (fc.n_heads / fc.n_kv_heads != 1 && fc.n_heads / fc.n_kv_heads != 2 && fc.n_heads / fc.n_kv_heads != 4 &&
         fc.n_heads / fc.n_kv_heads != 8))
        return set_error(AAEDN_EINVAL,
                         "aaedn_model_create: need dim, n_heads*head_dim, ffn_dim multiples of 32, head_dim a "
                         "multiple of 16 (<= %d), n_heads / n_kv_heads in {1, 2, 4, 8}",
                         ATTN_MAX_HD);
    // dim <= 16384: the lm_head ring holds x and at least two rows
    if (fc.dim > 16384 || fc.ffn_dim > 32768 || fc.max_seq > (1u << 20))
        return set_error(AAEDN_EINVAL, "aaedn_model_create: dimension too large (dim <= 16384, ffn_dim <= 32768)");
    aaedn_tp_plan plan{};
    {
        const int prc = aaedn_tp_plan_get(&fc, tp_rank, tp_size, &plan);
        if (prc)
            return prc;
    }
    // this rank's dims: heads, kv heads, ffn rows, lm_head rows
    aaedn_model_config lc = fc;
    lc.n_heads = plan.n_heads;
    lc.n_kv_heads = plan.n_kv_heads;
    lc.ffn_dim = plan.ffn_dim;
    lc.vocab = plan.vocab;
    aaedn_model* m = new aaedn_model();
    m->cfg = lc;
    m->full = fc;
    m->tp_rank = (int)tp_rank;
    m->tp_size = (int)tp_size;
    m->v0 = plan.vocab0;
    m->kpo = plan.o_k;
    m->kpd = plan.down_k;
    const aaedn_model_config& c = m->cfg;
    {
        const char* e = std::getenv("AAEDN_PDL");
        m->pdl = !(e && e[0] == '0');
        const char* t = std::getenv("AAEDN_TILED");
        m->tiled = !(t && t[0] == '0');
        const char* h = std::getenv("AAEDN_L2HINT");
        m->l2_hint = !(h && h[0] == '0');
    }
    m->page_size = 64;
    m->n_pages = (int)((c.max_seq + m->page_size - 1) / m->page_size);
    if (max_seqs)
    {
        // batched: a pool of kv_tokens / page_size pages; a sequence's page
        // table holds up to max_seq tokens
        m->max_seqs = max_seqs;
        m->pt_stride = (uint32_t)m->n_pages;
        m->n_pages = (int)((kv_tokens + m->page_size - 1) / m->page_size);
    }
    // about two attention CTAs per SM (a CTA walks its token range in
    // batches, so any split count covers any context length)
    int per_sm = 2;
    if (const char* e = std::getenv("AAEDN_ATTN_CTAS_PER_SM"))
        per_sm = std::max(1, std::min(4, std::atoi(e)));
    int S = std::max(1, (per_sm * sm_count() + (int)c.n_kv_heads - 1) / (int)c.n_kv_heads);
    S = std::max(1, std::min<int>(S, (int)std::max<uint32_t>(1, c.max_seq / 8)));
    S = std::min(S, 16); // the decode kernel merges at most 16 splits
    m->attn_S = S;
    m->attn_max_tok = (int)((c.max_seq + S - 1) / S);
    // lm_head: one CTA per SM, each streaming one contiguous run of rows
    m->lm_rows = std::max(1, (int)((c.vocab + sm_count() - 1) / sm_count()));
    m->lm_ctas = (int)((c.vocab + m->lm_rows - 1) / m->lm_rows);
    {
        // rows that fit beside x; every consumer warp owns stages/consumers
        const int fit = (int)std::min<size_t>(LM_MAX_STAGES,
                                              (200 * 1024 - (size_t)c.dim * 4 - 1024) / ((size_t)c.dim * 4));
        m->lm_consumers = fit >= LM_CONSUMERS ? LM_CONSUMERS : (fit >= 4 ? 4 : (fit >= 2 ? 2 : 1));
        m->lm_stages = fit / m->lm_consumers * m->lm_consumers;
    }
    {
        // prefill through the tensor-core GEMM: every matrix in the tile-major
        // layout (K % 128, N % 16), one GPU, head_dim a multiple of 32
        const size_t D = c.dim, hd = c.head_dim, F = c.ffn_dim;
        const size_t qkv_rows = (size_t)(c.n_heads + 2 * c.n_kv_heads) * hd;
        const bool ok = m->tp_size == 1 && m->tiled && tiles_ok(qkv_rows, D) && tiles_ok(D, m->kpo) &&
                        tiles_ok(2 * F, D) && tiles_ok(D, m->kpd) && hd % 32 == 0 && hd <= 256;
        // 1024 tokens a chunk by default: GEMMs of M = 1024 keep the tensor
        // pipe busy (M = 2048: 58 % of the bf16 peak in the five-product
        // form, M = 128: 32 %) for about 200 MB of chunk buffers at 7B
        const char* pe = std::getenv("AAEDN_PREFILL_ROWS");
        const int rows = pe ? std::atoi(pe) : 1024;
        m->pf_rows = ok && rows > 1 ? (int)std::min<uint32_t>((uint32_t)rows, c.max_seq) : 0;
        if (max_seqs)
        {
            if (!ok)
            {
                delete m;
                return set_error(AAEDN_EUNSUPPORTED, "aaedn_model_create_batched: the model's matrices need the "
                                                     "tile-major layout (K %% 128, N %% 16) and head_dim %% 32");
            }
            // a batch of max_seqs rows goes through the same buffers
            m->pf_rows = std::max<int>(std::max(m->pf_rows, 2), (int)max_seqs);
        }
    }
    const size_t bytes = plan_arena(m, false);
    cudaError_t e = cudaMalloc(reinterpret_cast<void**>(&m->arena), bytes);
    if (e != cudaSuccess)
    {
        delete m;
        return set_error(e == cudaErrorMemoryAllocation ? AAEDN_ENOMEM : AAEDN_ECUDA,
                         "aaedn_model_create: device arena of %zu bytes: %s", bytes, cudaGetErrorString(e));
    }
    m->arena_bytes = bytes;
    plan_arena(m, true);
    int rc = AAEDN_OK;
    auto fail = [&](int code) {
        aaedn_model_destroy(m);
        return code;
    };
    if (cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking) != cudaSuccess)
        return fail(set_error(AAEDN_ECUDA, "stream creation failed"));
    if (cudaMallocHost(reinterpret_cast<void**>(&m->pinned), ((size_t)c.max_seq + 16) * 4) != cudaSuccess)
        return fail(set_error(AAEDN_ENOMEM, "pinned staging allocation failed"));
    if (m->max_seqs)
    {
        if (cudaMallocHost(reinterpret_cast<void**>(&m->pinned_b), (size_t)m->max_seqs * 3 * 4) != cudaSuccess)
            return fail(set_error(AAEDN_ENOMEM, "pinned staging allocation failed"));
        m->seqs.assign(m->max_seqs, aaedn_model::Seq{});
        m->page_ref.assign((size_t)m->n_pages, 0);
        m->free_pages.resize((size_t)m->n_pages);
        for (int i = 0; i < m->n_pages; ++i)
            m->free_pages[(size_t)i] = m->n_pages - 1 - i; // handed out from the back: page 0 first
        m->h_pt.assign((size_t)m->max_seqs * m->pt_stride, 0);
    }
    if (cudaMemset(m->arena, 0, bytes) != cudaSuccess)
        return fail(set_error(AAEDN_ECUDA, "arena clear failed"));
    // RoPE tables (D3) and the identity page table of the single sequence
    std::vector<float> cs((size_t)c.max_seq * (c.head_dim / 2)), sn(cs.size());
    rc = aaedn_rope_table(cs.data(), sn.data(), c.max_seq, c.head_dim, (double)c.rope_theta, 1);
    if (rc)
        return fail(rc);
    std::vector<int> pt(m->n_pages);
    for (int i = 0; i < m->n_pages; ++i)
        pt[i] = i;
    std::vector<float> ones(c.dim, 1.0f);
    if (cudaMemcpy(m->rope_cos, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(m->rope_sin, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(m->page_table, pt.data(), pt.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(m->final_norm, ones.data(), c.dim * 4, cudaMemcpyHostToDevice) != cudaSuccess)
        return fail(set_error(AAEDN_ECUDA, "table upload failed"));
    for (auto& L : m->layers)
        if (cudaMemcpy(L.attn_norm, ones.data(), c.dim * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
            cudaMemcpy(L.ffn_norm, ones.data(), c.dim * 4, cudaMemcpyHostToDevice) != cudaSuccess)
            return fail(set_error(AAEDN_ECUDA, "norm upload failed"));
    // one process-wide value that covers every model (lm_smem_bytes <= 200 KB)
    if (cudaFuncSetAttribute(lm_head_argmax_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024) !=
        cudaSuccess)
        return fail(set_error(AAEDN_ECUDA, "lm_head smem attribute failed"));
    rc = attn_set_attrs<1>();
    if (rc)
        return fail(rc);
    {
        // decode attention as clusters of Sc splits per kv head (a power of
        // two <= 8 by default, <= max_seq / 8) merging in distributed shared
        // memory, when this GPU can hold such a cluster (7B, one B200: 8
        // splits 562 tok/s, 16 splits 520, the global merge over 10 splits
        // 552); AAEDN_ATTN_CLUSTER=0 keeps the global merge, =n caps Sc at n
        const char* ce = std::getenv("AAEDN_ATTN_CLUSTER");
        int cap = ce ? std::atoi(ce) : 8;
        int Sc = 16;
        while (Sc > 1 && (Sc > cap || Sc > (int)(c.max_seq / 8)))
            Sc >>= 1;
        const int G = (int)(c.n_heads / c.n_kv_heads);
        if (Sc >= 2 && attn_cluster_capacity(G, (int)c.head_dim, Sc, (int)c.n_kv_heads) >= 1)
            m->attn_cS = Sc;
        // more warps a CTA for MHA at head_dim <= 128, so one batch of K/V
        // loads covers more context (10: three CTAs per SM; AAEDN_ATTN_WARPS=8
        // keeps 8), only when every kv head's cluster can be resident at once.
        // 7B, one B200: 8 warps 682 tok/s, 10 warps 685-690 (16 warps, two
        // CTAs per SM: 620, clusters placed late)
        const char* we = std::getenv("AAEDN_ATTN_WARPS");
        const int nw = we ? std::atoi(we) : 10;
        if (m->attn_cS && nw == 10 && G == 1 && c.head_dim <= 128 &&
            attn_cluster_capacity(G, (int)c.head_dim, Sc, (int)c.n_kv_heads, nw) >= (int)c.n_kv_heads)
            m->attn_warps = nw;
    }
    rc = set_model_kernel_attrs();
    if (rc)
        return fail(rc);
    if (m->tp_size > 1)
        for (const DevLayer& L : m->layers)
            if (!(L.tqkv && L.to && L.tgu && L.td))
                return fail(set_error(AAEDN_EUNSUPPORTED, "tensor parallel decode needs every matrix tile-major"));
    *out = m;
    return AAEDN_OK;
}

extern "C" int aaedn_model_create(const aaedn_model_config* cfg, aaedn_model** out)
{
    return create_impl(cfg, 0, 1, out);
}

extern "C" int aaedn_model_create_tp(const aaedn_model_config* cfg, uint32_t tp_rank, uint32_t tp_size,
                                     aaedn_model** out)
{
    int rc = create_impl(cfg, tp_rank, tp_size, out);
    if (rc || tp_size == 1)
        return rc;
    aaedn_model* m = *out;
    // the peer-visible region: receive buffers [TP_MAX sources][2][dim],
    // flags [TP_MAX][4], argmax slots [TP_MAX] (one cudaMalloc: an IPC handle
    // covers it)
    const size_t part = (size_t)m->cfg.dim * 4;
    m->tp_region_bytes = (size_t)TP_MAX * 2 * part + TP_MAX * 16 + TP_MAX * 8 + 256;
    if (cudaMalloc(reinterpret_cast<void**>(&m->tp_region), m->tp_region_bytes) != cudaSuccess ||
        cudaMemset(m->tp_region, 0, m->tp_region_bytes) != cudaSuccess)
    {
        aaedn_model_destroy(m);
        *out = nullptr;
        return set_error(AAEDN_ENOMEM, "aaedn_model_create_tp: peer region");
    }
    m->tp.rank = (int)tp_rank;
    m->tp.size = (int)tp_size;
    return AAEDN_OK;
}

// addresses inside a rank's region
static void tp_layout(uint8_t* base, size_t dim, float*& recv, unsigned*& flags, float2*& best)
{
    recv = reinterpret_cast<float*>(base);
    flags = reinterpret_cast<unsigned*>(base + (size_t)TP_MAX * 2 * dim * 4);
    best = reinterpret_cast<float2*>(base + (size_t)TP_MAX * 2 * dim * 4 + TP_MAX * 16);
}

extern "C" int aaedn_model_tp_handle(aaedn_model* m, uint8_t* h_handle)
{
    MODEL_OK(m);
    if (m->tp_size < 2 || !h_handle)
        return set_error(AAEDN_EINVAL, "aaedn_model_tp_handle: not a tensor-parallel model or null output");
    cudaIpcMemHandle_t h;
    AAEDN_CUDA_TRY(cudaIpcGetMemHandle(&h, m->tp_region));
    static_assert(sizeof(h) == AAEDN_TP_HANDLE_BYTES, "IPC handle size");
    std::memcpy(h_handle, &h, sizeof h);
    return AAEDN_OK;
}

extern "C" int aaedn_model_tp_connect(aaedn_model* m, const uint8_t* h_handles)
{
    MODEL_OK(m);
    if (m->tp_size < 2 || !h_handles)
        return set_error(AAEDN_EINVAL, "aaedn_model_tp_connect: not a tensor-parallel model or null handles");
    if (m->tp_ready)
        return AAEDN_OK;
    const size_t dim = m->cfg.dim;
    for (int r = 0; r < m->tp_size; ++r)
    {
        uint8_t* base = m->tp_region;
        if (r != m->tp_rank)
        {
            cudaIpcMemHandle_t h;
            std::memcpy(&h, h_handles + (size_t)r * AAEDN_TP_HANDLE_BYTES, sizeof h);
            void* p = nullptr;
            AAEDN_CUDA_TRY(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
            m->tp_peer[r] = p;
            base = static_cast<uint8_t*>(p);
        }
        tp_layout(base, dim, m->tp.recv[r], m->tp.flags[r], m->tp.best[r]);
    }
    m->tp.my_flags = m->tp.flags[m->tp_rank];
    m->tp.dim = (int)dim;
    m->tp_ready = true;
    return AAEDN_OK;
}

extern "C" int aaedn_model_destroy(aaedn_model* m)
{
    if (!m)
        return AAEDN_OK;
    if (m->stream)
        cudaStreamSynchronize(m->stream);
    if (m->graph_exec)
        cudaGraphExecDestroy(m->graph_exec);
    for (int r = 0; r < TP_MAX; ++r)
        if (m->tp_peer[r])
            cudaIpcCloseMemHandle(m->tp_peer[r]);
    if (m->tp_region)
        cudaFree(m->tp_region);
    if (m->arena)
        cudaFree(m->arena);
    if (m->pinned)
        cudaFreeHost(m->pinned);
    if (m->pinned_b)
        cudaFreeHost(m->pinned_b);
    if (m->stream)
        cudaStreamDestroy(m->stream);
    delete m;
    return AAEDN_OK;
}

extern "C" int aaedn_model_config_get(const aaedn_model* m, aaedn_model_config* out)
{
    MODEL_OK(m);
    if (!out)
        return set_error(AAEDN_EINVAL, "null output");
    *out = m->full; // the model's dims (cfg holds this rank's share)
    return AAEDN_OK;
}

extern "C" void* aaedn_model_stream(aaedn_model* m) { return m ? (void*)m->stream : nullptr; }
extern "C" size_t aaedn_model_arena_bytes(const aaedn_model* m) { return m ? m->arena_bytes : 0; }
extern "C" uint32_t aaedn_model_pos(aaedn_model* m) { return m ? m->h_pos : 0; }
extern "C" uint32_t aaedn_model_prefill_rows(const aaedn_model* m) { return m ? (uint32_t)m->pf_rows : 0u; }

// ---- fused_matmul on tile-major weights (the model's engines) ------------

extern "C" size_t aaedn_q4_tiled_bytes(size_t N, size_t K) { return tiled_bytes(N, K); }

extern "C" int aaedn_q4_repack_tiled(const uint8_t* h_codes, const uint16_t* h_scales, size_t N, size_t K,
                                     uint8_t* h_out)
{
    if (!h_codes || !h_scales || !h_out)
        return set_error(AAEDN_EINVAL, "aaedn_q4_repack_tiled: null buffer");
    if (N % 16 || K % 128 || K == 0)
        return set_error(AAEDN_EINVAL, "aaedn_q4_repack_tiled: N %% 16 and K %% 128 must be 0 (N %zu, K %zu)", N, K);
    repack_tiled(h_codes, h_scales, N, K, h_out);
    return AAEDN_OK;
}

extern "C" int aaedn_cu_fused_matmul_tiled(const float* d_in, const uint8_t* d_tiled, float* d_out, size_t M,
                                           size_t N, size_t K, void* stream)
{
    if (M == 0 || N == 0 || K == 0)
        return AAEDN_OK;
    if (!d_in || !d_tiled || !d_out)
        return set_error(AAEDN_EINVAL, "aaedn_cu_fused_matmul_tiled: null buffer");
    if (!tiles_ok(N, K) || M > (size_t)INT32_MAX || N > (size_t)INT32_MAX)
        return set_error(AAEDN_EINVAL, "aaedn_cu_fused_matmul_tiled: N %% 16, K %% 128 must be 0 and K <= 32768");
    if ((reinterpret_cast<uintptr_t>(d_tiled) | reinterpret_cast<uintptr_t>(d_in)) & 15)
        return set_error(AAEDN_EINVAL, "aaedn_cu_fused_matmul_tiled: buffers must be 16-byte aligned");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    static PerDeviceOnce attrs;
    int rc = attrs.run([]() { return set_gemv_attrs<PRO_PLAIN, EPI_STORE>(); });
    if (rc)
        return rc;
    if (M == 1)
    {
        // the decode GEMV engine
        GemvParams p{};
        p.w = d_tiled;
        p.N = (int)N;
        p.K = (int)K;
        p.x = d_in;
        p.lda = K;
        p.y = d_out;
        p.ldc = N;
        p.l2_hint = 1;
        return model_gemv<PRO_PLAIN, EPI_STORE>(p, st, false, true);
    }
    // more rows: the tcgen05 GEMM over the same layout
    TcGemmArgs a{};
    a.x = d_in;
    a.lda = K;
    a.M = (int)M;
    a.N = (int)N;
    a.K = (int)K;
    a.w = d_tiled;
    a.w_layout = TC_W_TILED;
    a.out = d_out;
    a.ldc = N;
    a.err = tc_api_err_word();
    if (!a.err)
        return set_error(AAEDN_ECUDA, "aaedn_cu_fused_matmul_tiled: error word allocation failed");
    a.workspace_bytes = tc_gemm_workspace_bytes(a.M, a.N, a.K);
    AAEDN_CUDA_TRY(cudaMallocAsync(&a.workspace, a.workspace_bytes, st));
    rc = tc_gemm(a, st);
    AAEDN_CUDA_TRY(cudaFreeAsync(a.workspace, st));
    return rc;
}

extern "C" uint32_t aaedn_model_kernels_per_step(const aaedn_model* m)
{
    return m ? 5u * m->cfg.n_layers + 1u : 0u;
}

// Device row r of a rope-paired head block holds logical row
// 8j + r (r < 8) or half + 8j + r - 8 (r >= 8), j = r_in_head / 16.
static inline size_t rope_pair_row(size_t r_in_head, size_t hd)
{
    const size_t j = r_in_head / 16, r = r_in_head % 16;
    return r < 8 ? 8 * j + r : hd / 2 + 8 * j + (r - 8);
}

// Uploads one matrix (row-major host codes/scales, rows already in device
// order) into its region: tile-major when the layer says so.
static int upload_matrix(uint8_t* dw, uint16_t* ds, bool tiled, const uint8_t* codes, const uint16_t* scales,
                         size_t N, size_t K)
{
    if (tiled)
    {
        std::vector<uint8_t> blob(tiled_bytes(N, K));
        repack_tiled(codes, scales, N, K, blob.data());
        AAEDN_CUDA_TRY(cudaMemcpy(dw, blob.data(), blob.size(), cudaMemcpyHostToDevice));
        return AAEDN_OK;
    }
    AAEDN_CUDA_TRY(cudaMemcpy(dw, codes, N * K / 2, cudaMemcpyHostToDevice));
    AAEDN_CUDA_TRY(cudaMemcpy(ds, scales, N * K / 32 * 2, cudaMemcpyHostToDevice));
    return AAEDN_OK;
}

// Copies columns [col0, col0 + ncols) of source row srow (Ks columns) into
// device-order row drow of a Kd-column matrix (the rest of the row stays
// zero: padding). Columns come in whole 32-blocks.
static void copy_row(std::vector<uint8_t>& dd, std::vector<uint16_t>& ds, size_t drow, size_t Kd, const uint8_t* sd,
                     const uint16_t* ss, size_t srow, size_t Ks, size_t col0, size_t ncols)
{
    std::memcpy(dd.data() + drow * Kd / 2, sd + srow * Ks / 2 + col0 / 2, ncols / 2);
    std::memcpy(ds.data() + drow * Kd / 32, ss + srow * Ks / 32 + col0 / 32, ncols / 32 * 2);
}

// Weights arrive whole (the model's dims); a tensor-parallel rank keeps its
// share: q rows of its heads, k/v rows of its kv heads, gate/up rows
// [r F/T, (r+1) F/T), and the matching input columns of o and down (padded
// to kpo / kpd with zero columns).
extern "C" int aaedn_model_set_layer(aaedn_model* m, uint32_t layer, const aaedn_layer_host* w)
{
    MODEL_OK(m);
    if (!w || layer >= m->cfg.n_layers)
        return set_error(AAEDN_EINVAL, "aaedn_model_set_layer: bad layer or null weights");
    if (!w->wq || !w->wk || !w->wv || !w->wo || !w->wg || !w->wu || !w->wd || !w->sq || !w->sk || !w->sv || !w->so ||
        !w->sg || !w->su || !w->sd)
        return set_error(AAEDN_EINVAL, "aaedn_model_set_layer: null tensor");
    const aaedn_model_config& c = m->cfg; // this rank's share
    const size_t D = c.dim, hd = c.head_dim, H = c.n_heads, KV = c.n_kv_heads, F = c.ffn_dim;
    const size_t Hf = m->full.n_heads, Ff = m->full.ffn_dim;
    const size_t r = (size_t)m->tp_rank;
    const size_t q0 = r * H * hd, k0 = r * KV * hd, f0 = r * F; // first source row / column of the share
    const DevLayer& L = m->layers[layer];
    AAEDN_CUDA_TRY(cudaStreamSynchronize(m->stream));
    {
        const size_t rows = (H + 2 * KV) * hd;
        std::vector<uint8_t> dd(rows * D / 2);
        std::vector<uint16_t> ds(rows * D / 32);
        for (size_t dr = 0; dr < rows; ++dr)
        {
            if (dr < H * hd)
                copy_row(dd, ds, dr, D, w->wq, w->sq, q0 + (dr / hd) * hd + rope_pair_row(dr % hd, hd), D, 0, D);
            else if (dr < (H + KV) * hd)
            {
                const size_t rel = dr - H * hd;
                copy_row(dd, ds, dr, D, w->wk, w->sk, k0 + (rel / hd) * hd + rope_pair_row(rel % hd, hd), D, 0, D);
            }
            else
                copy_row(dd, ds, dr, D, w->wv, w->sv, k0 + dr - (H + KV) * hd, D, 0, D);
        }
        int rc = upload_matrix(L.wqkv, L.sqkv, L.tqkv, dd.data(), ds.data(), rows, D);
        if (rc)
            return rc;
    }
    {
        std::vector<uint8_t> dd(D * m->kpo / 2, 0);
        std::vector<uint16_t> ds(D * m->kpo / 32, 0);
        for (size_t n = 0; n < D; ++n)
            copy_row(dd, ds, n, m->kpo, w->wo, w->so, n, Hf * hd, q0, H * hd);
        int rc = upload_matrix(L.wo, L.so, L.to, dd.data(), ds.data(), D, m->kpo);
        if (rc)
            return rc;
    }
    {
        const size_t rows = 2 * F;
        std::vector<uint8_t> dd(rows * D / 2);
        std::vector<uint16_t> ds(rows * D / 32);
        for (size_t dr = 0; dr < rows; ++dr)
        {
            const size_t j = dr / 16, rr = dr % 16;
            if (rr < 8)
                copy_row(dd, ds, dr, D, w->wg, w->sg, f0 + 8 * j + rr, D, 0, D);
            else
                copy_row(dd, ds, dr, D, w->wu, w->su, f0 + 8 * j + rr - 8, D, 0, D);
        }
        int rc = upload_matrix(L.wgu, L.sgu, L.tgu, dd.data(), ds.data(), rows, D);
        if (rc)
            return rc;
    }
    {
        std::vector<uint8_t> dd(D * m->kpd / 2, 0);
        std::vector<uint16_t> ds(D * m->kpd / 32, 0);
        for (size_t n = 0; n < D; ++n)
            copy_row(dd, ds, n, m->kpd, w->wd, w->sd, n, Ff, f0, F);
        int rc = upload_matrix(L.wd, L.sd, L.td, dd.data(), ds.data(), D, m->kpd);
        if (rc)
            return rc;
    }
    if (w->attn_norm)
        AAEDN_CUDA_TRY(cudaMemcpy(L.attn_norm, w->attn_norm, D * 4, cudaMemcpyHostToDevice));
    if (w->ffn_norm)
        AAEDN_CUDA_TRY(cudaMemcpy(L.ffn_norm, w->ffn_norm, D * 4, cudaMemcpyHostToDevice));
    return AAEDN_OK;
}

extern "C" int aaedn_model_set_globals(aaedn_model* m, const float* h_embedding, const float* h_final_norm,
                                       const float* h_lm_head)
{
    MODEL_OK(m);
    const aaedn_model_config& c = m->cfg;
    AAEDN_CUDA_TRY(cudaStreamSynchronize(m->stream));
    if (h_embedding)
        AAEDN_CUDA_TRY(
            cudaMemcpy(m->embedding, h_embedding, (size_t)m->full.vocab * c.dim * 4, cudaMemcpyHostToDevice));
    if (h_final_norm)
        AAEDN_CUDA_TRY(cudaMemcpy(m->final_norm, h_final_norm, (size_t)c.dim * 4, cudaMemcpyHostToDevice));
    if (h_lm_head) // the whole matrix in; this rank keeps rows [v0, v0 + its share)
        AAEDN_CUDA_TRY(cudaMemcpy(m->lm_head, h_lm_head + (size_t)m->v0 * c.dim, (size_t)c.vocab * c.dim * 4,
                                  cudaMemcpyHostToDevice));
    return AAEDN_OK;
}

extern "C" int aaedn_model_synthesize(aaedn_model* m, uint64_t seed)
{
    MODEL_OK(m);
    const aaedn_model_config& c = m->full; // whole tensors: set_layer keeps this rank's share
    const size_t D = c.dim, hd = c.head_dim, H = c.n_heads, KV = c.n_kv_heads, F = c.ffn_dim, V = c.vocab;
    struct Mat
    {
        size_t rows, cols;
        std::vector<uint8_t> d;
        std::vector<uint16_t> s;
    };
    Mat mats[7] = {{H * hd, D, {}, {}}, {KV * hd, D, {}, {}}, {KV * hd, D, {}, {}}, {D, H * hd, {}, {}},
                   {F, D, {}, {}},      {F, D, {}, {}},       {D, F, {}, {}}};
    std::vector<float> buf;
    for (uint32_t l = 0; l < c.n_layers; ++l)
    {
        for (int i = 0; i < 7; ++i)
        {
            const size_t n = mats[i].rows * mats[i].cols;
            buf.resize(n);
            aaedn_host::synth_normal(seed, 16 + 8ull * l + (uint64_t)i, 0.02f, buf.data(), n);
            mats[i].d.assign((n + 1) / 2, 0);
            mats[i].s.assign((n + 31) / 32, 0);
            aaedn_host::quantize_q4(buf.data(), n, mats[i].d.data(), mats[i].s.data());
        }
        aaedn_layer_host w{};
        w.wq = mats[0].d.data();
        w.sq = mats[0].s.data();
        w.wk = mats[1].d.data();
        w.sk = mats[1].s.data();
        w.wv = mats[2].d.data();
        w.sv = mats[2].s.data();
        w.wo = mats[3].d.data();
        w.so = mats[3].s.data();
        w.wg = mats[4].d.data();
        w.sg = mats[4].s.data();
        w.wu = mats[5].d.data();
        w.su = mats[5].s.data();
        w.wd = mats[6].d.data();
        w.sd = mats[6].s.data();
        int rc = aaedn_model_set_layer(m, l, &w);
        if (rc)
            return rc;
    }
    buf.assign(V * D, 0.0f);
    aaedn_host::synth_normal(seed, 0, 0.02f, buf.data(), V * D);
    int rc = aaedn_model_set_globals(m, buf.data(), nullptr, nullptr);
    if (rc)
        return rc;
    aaedn_host::synth_normal(seed, 1, 0.02f, buf.data(), V * D);
    return aaedn_model_set_globals(m, nullptr, nullptr, buf.data());
}

extern "C" int aaedn_model_reset(aaedn_model* m)
{
    MODEL_OK(m);
    AAEDN_CUDA_TRY(cudaStreamSynchronize(m->stream));
    AAEDN_CUDA_TRY(cudaMemsetAsync(m->state, 0, sizeof(DecodeState), m->stream));
    AAEDN_CUDA_TRY(cudaStreamSynchronize(m->stream));
    m->h_pos = 0;
    return AAEDN_OK;
}

extern "C" int aaedn_model_forward(aaedn_model* m, const uint32_t* h_tokens, size_t n, float* h_logits)
{
    MODEL_OK(m);
    if (m->max_seqs)
        return set_error(AAEDN_EUNSUPPORTED, "a batched model steps its sequences with aaedn_model_step_batch");
    const aaedn_model_config& c = m->cfg;
    const uint32_t V = m->full.vocab;
    if (n == 0 || !h_tokens) // src/transformer.cpp:130-135: zero logits
    {
        if (h_logits)
            std::memset(h_logits, 0, (size_t)V * 4);
        return AAEDN_OK;
    }
    for (size_t i = 0; i < n; ++i)
        if (h_tokens[i] >= V) // src/transformer.cpp:137-142
        {
            if (h_logits)
                std::memset(h_logits, 0, (size_t)V * 4);
            return set_error(AAEDN_EINVAL, "token id %u >= vocab %u", h_tokens[i], V);
        }
    if ((size_t)m->h_pos + n > c.max_seq)
        return set_error(AAEDN_ESTATE, "sequence full: pos %u + %zu > max_seq %u", m->h_pos, n, c.max_seq);
    int rc = put_tokens(m, h_tokens, n);
    if (!rc)
        rc = write_state(m, m->h_pos, m->h_pos + (uint32_t)n);
    if (!rc)
        rc = (n > 1 && m->pf_rows) ? prefill(m, n) : run_steps(m, n);
    if (rc)
        return rc;
    m->h_pos += (uint32_t)n;
    if (h_logits) // a tensor-parallel rank fills its own vocabulary slice
        AAEDN_CUDA_TRY(cudaMemcpyAsync(h_logits + m->v0, m->logits, (size_t)c.vocab * 4, cudaMemcpyDeviceToHost,
                                       m->stream));
    return device_status(m);
}

extern "C" int aaedn_model_generate(aaedn_model* m, const uint32_t* h_prompt, size_t n_prompt, size_t n_new,
                                    uint32_t* h_out)
{
    MODEL_OK(m);
    if (m->max_seqs)
        return set_error(AAEDN_EUNSUPPORTED, "a batched model steps its sequences with aaedn_model_step_batch");
    const aaedn_model_config& c = m->cfg;
    if (!h_prompt || n_prompt == 0 || (n_new && !h_out))
        return set_error(AAEDN_EINVAL, "aaedn_model_generate: empty prompt or null output");
    for (size_t i = 0; i < n_prompt; ++i)
        if (h_prompt[i] >= m->full.vocab)
            return set_error(AAEDN_EINVAL, "token id %u >= vocab %u", h_prompt[i], m->full.vocab);
    const size_t steps = n_prompt + (n_new ? n_new - 1 : 0);
    if ((size_t)m->h_pos + steps > c.max_seq)
        return set_error(AAEDN_ESTATE, "sequence full: pos %u + %zu steps > max_seq %u", m->h_pos, steps, c.max_seq);
    int rc = put_tokens(m, h_prompt, n_prompt);
    if (!rc)
        rc = write_state(m, m->h_pos, m->h_pos + (uint32_t)n_prompt);
    if (!rc && n_prompt > 1 && m->pf_rows)
    {
        // the prompt through the tensor-core prefill, then the decode steps
        rc = prefill(m, n_prompt);
        if (!rc)
        {
            m->h_pos += (uint32_t)n_prompt;
            rc = run_steps(m, steps - n_prompt);
            if (!rc)
                m->h_pos += (uint32_t)(steps - n_prompt);
        }
    }
    else if (!rc)
    {
        rc = run_steps(m, steps);
        if (!rc)
            m->h_pos += (uint32_t)steps;
    }
    if (rc)
        return rc;
    if (n_new)
        AAEDN_CUDA_TRY(cudaMemcpyAsync(h_out, m->out_tokens, n_new * 4, cudaMemcpyDeviceToHost, m->stream));
    return device_status(m);
}

extern "C" int aaedn_model_decode_steps(aaedn_model* m, size_t n_steps)
{
    MODEL_OK(m);
    if (m->max_seqs)
        return set_error(AAEDN_EUNSUPPORTED, "a batched model steps its sequences with aaedn_model_step_batch");
    if (m->h_pos == 0)
        return set_error(AAEDN_ESTATE, "aaedn_model_decode_steps: no token in the sequence yet");
    if ((size_t)m->h_pos + n_steps > m->cfg.max_seq)
        return set_error(AAEDN_ESTATE, "sequence full: pos %u + %zu > max_seq %u", m->h_pos, n_steps, m->cfg.max_seq);
    int rc = run_steps(m, n_steps);
    if (rc)
        return rc;
    m->h_pos += (uint32_t)n_steps;
    return AAEDN_OK;
}

extern "C" int aaedn_model_logits(aaedn_model* m, float* h_logits)
{
    MODEL_OK(m);
    if (!h_logits)
        return set_error(AAEDN_EINVAL, "null output");
    AAEDN_CUDA_TRY(cudaMemcpyAsync(h_logits + m->v0, m->logits, (size_t)m->cfg.vocab * 4, cudaMemcpyDeviceToHost,
                                   m->stream));
    AAEDN_CUDA_TRY(cudaStreamSynchronize(m->stream));
    return AAEDN_OK;
}

extern "C" int aaedn_model_tokens(aaedn_model* m, uint32_t* h_out, size_t n)
{
    MODEL_OK(m);
    if (n > m->cfg.max_seq || (n && !h_out))
        return set_error(AAEDN_EINVAL, "aaedn_model_tokens: bad count");
    if (n)
        AAEDN_CUDA_TRY(cudaMemcpyAsync(h_out, m->out_tokens, n * 4, cudaMemcpyDeviceToHost, m->stream));
    AAEDN_CUDA_TRY(cudaStreamSynchronize(m->stream));
    return AAEDN_OK;
}

extern "C" int aaedn_model_forward_debug(aaedn_model* m, uint32_t token, float* h_hidden, float* h_logits)
{
    MODEL_OK(m);
    if (m->max_seqs)
        return set_error(AAEDN_EUNSUPPORTED, "a batched model steps its sequences with aaedn_model_step_batch");
    if (m->tp_size > 1) // the residual of a layer is complete only inside the next layer's kernels
        return set_error(AAEDN_EUNSUPPORTED, "aaedn_model_forward_debug: not for tensor-parallel models");
    const aaedn_model_config& c = m->cfg;
    if (token >= m->full.vocab)
        return set_error(AAEDN_EINVAL, "token id %u >= vocab %u", token, m->full.vocab);
    if (m->h_pos + 1 > c.max_seq)
        return set_error(AAEDN_ESTATE, "sequence full");
    int rc = put_tokens(m, &token, 1);
    if (!rc)
        rc = write_state(m, m->h_pos, m->h_pos + 1);
    if (!rc)
        rc = enqueue_step(m, m->stream, true);
    if (rc)
        return rc;
    m->h_pos += 1;
    if (h_hidden)
        AAEDN_CUDA_TRY(cudaMemcpyAsync(h_hidden, m->dbg_hidden, (size_t)c.n_layers * c.dim * 4,
                                       cudaMemcpyDeviceToHost, m->stream));
    if (h_logits)
        AAEDN_CUDA_TRY(
            cudaMemcpyAsync(h_logits + m->v0, m->logits, (size_t)c.vocab * 4, cudaMemcpyDeviceToHost, m->stream));
    AAEDN_CUDA_TRY(cudaStreamSynchronize(m->stream));
    return AAEDN_OK;
}

extern "C" int aaedn_model_rewind(aaedn_model* m, uint32_t pos)
{
    MODEL_OK(m);
    if (pos == 0 || pos > m->h_pos)
        return set_error(AAEDN_EINVAL, "aaedn_model_rewind: pos %u outside [1, %u]", pos, m->h_pos);
    AAEDN_CUDA_TRY(cudaStreamSynchronize(m->stream));
    // inputs from here on are the greedy tokens: n_prompt <= pos
    int rc = write_state(m, pos, pos);
    if (rc)
        return rc;
    AAEDN_CUDA_TRY(cudaStreamSynchronize(m->stream));
    m->h_pos = pos;
    return AAEDN_OK;
}

extern "C" int aaedn_model_profile_step(aaedn_model* m, float* h_ms, uint32_t cap, uint32_t* n_out)
{
    MODEL_OK(m);
    const uint32_t nk = aaedn_model_kernels_per_step(m);
    if (n_out)
        *n_out = nk;
    if (!h_ms || cap < nk)
        return set_error(AAEDN_EINVAL, "aaedn_model_profile_step: need room for %u timings", nk);
    if (m->h_pos == 0 || m->h_pos + 1 > m->cfg.max_seq)
        return set_error(AAEDN_ESTATE, "aaedn_model_profile_step: sequence empty or full");
    std::vector<cudaEvent_t> ev(nk + 1, nullptr);
    for (auto& e : ev)
        AAEDN_CUDA_TRY(cudaEventCreate(&e));
    auto cleanup = [&]() {
        for (auto& e : ev)
            if (e)
                cudaEventDestroy(e);
    };
    // one replay of a graph holding the step and its event records, so the
    // kernels run back to back as in the decode graph
    const uint64_t before = g_launches.load();
    cudaError_t e = cudaStreamBeginCapture(m->stream, cudaStreamCaptureModeThreadLocal);
    if (e != cudaSuccess)
    {
        cleanup();
        return set_error(AAEDN_ECUDA, "profile capture: %s", cudaGetErrorString(e));
    }
    int rc = enqueue_step(m, m->stream, false, &ev);
    cudaGraph_t g = nullptr;
    e = cudaStreamEndCapture(m->stream, &g);
    g_launches.fetch_sub(g_launches.load() - before);
    cudaGraphExec_t ex = nullptr;
    if (!rc && e == cudaSuccess)
        e = cudaGraphInstantiate(&ex, g, 0);
    if (g)
        cudaGraphDestroy(g);
    if (!rc && e == cudaSuccess)
        e = cudaGraphLaunch(ex, m->stream);
    if (!rc && e == cudaSuccess)
        e = cudaStreamSynchronize(m->stream);
    if (ex)
        cudaGraphExecDestroy(ex);
    if (!rc && e == cudaSuccess)
    {
        count_launch(nk);
        for (uint32_t i = 0; i < nk && e == cudaSuccess; ++i)
            e = cudaEventElapsedTime(&h_ms[i], ev[i], ev[i + 1]);
    }
    cleanup();
    if (rc)
        return rc;
    if (e != cudaSuccess)
        return set_error(AAEDN_ECUDA, "profile step: %s", cudaGetErrorString(e));
    m->h_pos += 1;
    return AAEDN_OK;
}

// Tracing: device time of sub-graphs of one decode step, each replayed
// `reps` times back to back (same launch setup as the decode graph).
// h_ms[i] = ms per step of: 0 all kernels, 1 the four dequant-GEMVs of every
// layer, 2 qkv, 3 attention, 4 o, 5 gate/up, 6 down, 7 lm_head. The KV cache
// and hidden state are left in an undefined state: rewind or reset after.
extern "C" int aaedn_model_profile_parts(aaedn_model* m, uint32_t reps, float* h_ms, uint32_t cap)
{
    MODEL_OK(m);
    if (m->tp_size > 1) // a part alone would wait for partials its peers never send
        return set_error(AAEDN_EUNSUPPORTED, "aaedn_model_profile_parts: not for tensor-parallel models");
    static const int masks[8] = {K_ALL, K_QKV | K_O | K_GU | K_DOWN, K_QKV, K_ATTN, K_O, K_GU, K_DOWN, K_LM};
    if (!h_ms || cap < 8 || reps == 0)
        return set_error(AAEDN_EINVAL, "aaedn_model_profile_parts: need 8 outputs and reps > 0");
    if (m->h_pos == 0 || (size_t)m->h_pos + reps + 2 > m->cfg.max_seq)
        return set_error(AAEDN_ESTATE, "aaedn_model_profile_parts: sequence empty or too full for %u replays", reps);
    AAEDN_CUDA_TRY(cudaStreamSynchronize(m->stream));
    cudaEvent_t e0 = nullptr, e1 = nullptr;
    AAEDN_CUDA_TRY(cudaEventCreate(&e0));
    AAEDN_CUDA_TRY(cudaEventCreate(&e1));
    int rc = AAEDN_OK;
    for (int i = 0; i < 8 && rc == AAEDN_OK; ++i)
    {
        // the step must not advance the position: keep pos fixed by restoring it
        const uint64_t before = g_launches.load();
        cudaGraph_t g = nullptr;
        cudaGraphExec_t ex = nullptr;
        cudaError_t e = cudaStreamBeginCapture(m->stream, cudaStreamCaptureModeThreadLocal);
        if (e == cudaSuccess)
        {
            rc = enqueue_step(m, m->stream, false, nullptr, masks[i]);
            e = cudaStreamEndCapture(m->stream, &g);
        }
        g_launches.fetch_sub(g_launches.load() - before);
        if (!rc && e == cudaSuccess)
            e = cudaGraphInstantiate(&ex, g, 0);
        if (g)
            cudaGraphDestroy(g);
        if (!rc && e == cudaSuccess)
            e = cudaGraphLaunch(ex, m->stream); // warm
        if (!rc && e == cudaSuccess)
            e = cudaEventRecord(e0, m->stream);
        for (uint32_t r = 0; r < reps && !rc && e == cudaSuccess; ++r)
            e = cudaGraphLaunch(ex, m->stream);
        if (!rc && e == cudaSuccess)
            e = cudaEventRecord(e1, m->stream);
        if (!rc && e == cudaSuccess)
            e = cudaEventSynchronize(e1);
        float ms = 0.0f;
        if (!rc && e == cudaSuccess)
            e = cudaEventElapsedTime(&ms, e0, e1);
        if (ex)
            cudaGraphExecDestroy(ex);
        if (!rc && e != cudaSuccess)
            rc = set_error(AAEDN_ECUDA, "profile parts: %s", cudaGetErrorString(e));
        h_ms[i] = ms / reps;
        // lm_head advanced the device position once per replay: put it back
        if (!rc && (masks[i] & K_LM))
            rc = write_state(m, m->h_pos, m->h_pos);
        if (!rc)
            rc = (cudaStreamSynchronize(m->stream) == cudaSuccess) ? AAEDN_OK
                                                                    : set_error(AAEDN_ECUDA, "profile sync");
    }
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    return rc;
}

extern "C" int aaedn_model_trace_kernels(aaedn_model* m, uint64_t* h_stamps, size_t cap, uint32_t* h_grid,
                                         size_t cap_grid)
{
    MODEL_OK(m);
    const aaedn_model_config& c = m->cfg;
    const size_t nk = (size_t)c.n_layers * 5 + 1, per = (size_t)STEP_TRACE_CTAS * STEP_TRACE_EVENTS;
    if (m->tp_size > 1)
        return set_error(AAEDN_EUNSUPPORTED, "aaedn_model_trace_kernels: not for a tensor-parallel model");
    if (!h_stamps || !h_grid || cap < nk * per || cap_grid < nk)
        return set_error(AAEDN_EINVAL, "aaedn_model_trace_kernels: need %zu stamps and %zu grid sizes", nk * per, nk);
    if (m->h_pos == 0 || (size_t)m->h_pos + 2 > c.max_seq)
        return set_error(AAEDN_ESTATE, "aaedn_model_trace_kernels: sequence empty or full");
    for (uint32_t l = 0; l < c.n_layers; ++l)
    {
        const DevLayer& L = m->layers[l];
        const GemvParams g[4] = {qkv_params(m, l), o_params(m, l), gu_params(m, l), down_params(m, l)};
        const bool t[4] = {L.tqkv, L.to, L.tgu, L.td};
        const int slot[4] = {0, 2, 3, 4};
        for (int i = 0; i < 4; ++i)
            h_grid[(size_t)l * 5 + slot[i]] =
                t[i] ? (uint32_t)std::min(g[i].N / 16, sm_count()) : 0u; // 0: not traced (row-major GEMV)
        h_grid[(size_t)l * 5 + 1] = (uint32_t)(c.n_kv_heads * (m->attn_cS ? m->attn_cS : m->attn_S));
    }
    h_grid[nk - 1] = (uint32_t)m->lm_ctas;
    unsigned long long* d = nullptr;
    AAEDN_CUDA_TRY(cudaStreamSynchronize(m->stream));
    AAEDN_CUDA_TRY(cudaMalloc(reinterpret_cast<void**>(&d), nk * per * 8));
    cudaGraph_t g = nullptr;
    cudaGraphExec_t ge = nullptr;
    int rc = AAEDN_OK;
    cudaError_t e = cudaMemsetAsync(d, 0, nk * per * 8, m->stream);
    if (e == cudaSuccess)
        e = cudaStreamBeginCapture(m->stream, cudaStreamCaptureModeThreadLocal);
    if (e == cudaSuccess)
    {
        rc = enqueue_step(m, m->stream, false, nullptr, K_ALL, d);
        e = cudaStreamEndCapture(m->stream, &g);
    }
    if (!rc && e == cudaSuccess)
        e = cudaGraphInstantiate(&ge, g, 0);
    if (!rc && e == cudaSuccess)
        e = cudaGraphLaunch(ge, m->stream);
    if (!rc && e == cudaSuccess)
        e = cudaMemcpyAsync(h_stamps, d, nk * per * 8, cudaMemcpyDeviceToHost, m->stream);
    if (!rc && e == cudaSuccess)
        e = cudaStreamSynchronize(m->stream);
    if (!rc && e != cudaSuccess)
        rc = set_error(AAEDN_ECUDA, "trace kernels: %s", cudaGetErrorString(e));
    if (ge)
        cudaGraphExecDestroy(ge);
    if (g)
        cudaGraphDestroy(g);
    cudaFree(d);
    if (!rc)
        rc = write_state(m, m->h_pos, m->h_pos); // the traced step does not count
    if (!rc && cudaStreamSynchronize(m->stream) != cudaSuccess)
        rc = set_error(AAEDN_ECUDA, "trace kernels sync");
    return rc;
}

extern "C" int aaedn_model_status(aaedn_model* m)
{
    MODEL_OK(m);
    return device_status(m);
}

extern "C" int aaedn_model_next_token(aaedn_model* m, uint32_t* h_token)
{
    MODEL_OK(m);
    if (!h_token)
        return set_error(AAEDN_EINVAL, "null output");
    uint32_t* w = m->pinned + m->cfg.max_seq + 5;
    AAEDN_CUDA_TRY(cudaMemcpyAsync(w, &m->state->next_token, 4, cudaMemcpyDeviceToHost, m->stream));
    AAEDN_CUDA_TRY(cudaStreamSynchronize(m->stream));
    *h_token = *w;
    return AAEDN_OK;
}

// ---------------------------------------------------------------------------
// Batched sequences over a shared, paged KV cache: the per-agent view of
// src/kvcache.cpp:15-60 (segment_tables[6], one per agent) and the branch
// protocol of docs/sdd.md:206-215 (diverge: the child continues from the
// parent's tokens; prune: the branch's storage is released) on the device.
// A sequence is a page table; fork copies the table (the pages are shared,
// counted), an append into a shared page copies that page first (copy on
// write), close releases the pages no other sequence holds.
// ---------------------------------------------------------------------------

#define BATCHED_OK(m)                                                                                         \
    do                                                                                                        \
    {                                                                                                         \
        MODEL_OK(m);                                                                                          \
        if (!(m)->max_seqs)                                                                                   \
            return set_error(AAEDN_EUNSUPPORTED, "not a batched model (aaedn_model_create_batched)");          \
    } while (0)

static int seq_ok(aaedn_model* m, uint32_t seq)
{
    if (seq >= m->max_seqs || !m->seqs[seq].open)
        return set_error(AAEDN_EINVAL, "sequence %u is not open", seq);
    return AAEDN_OK;
}

// Uploads sequence seq's row of the device page table.
static int upload_pt(aaedn_model* m, uint32_t seq)
{
    int* row = m->h_pt.data() + (size_t)seq * m->pt_stride;
    const auto& pg = m->seqs[seq].pages;
    std::fill(row, row + m->pt_stride, 0);
    std::copy(pg.begin(), pg.end(), row);
    // pageable source: the copy has read it when the call returns
    AAEDN_CUDA_TRY(cudaMemcpyAsync(m->seq_pt + (size_t)seq * m->pt_stride, row, (size_t)m->pt_stride * 4,
                                   cudaMemcpyHostToDevice, m->stream));
    return AAEDN_OK;
}

static void release_pages(aaedn_model* m, std::vector<int>& pages)
{
    for (int pg : pages)
        if (--m->page_ref[(size_t)pg] == 0)
            m->free_pages.push_back(pg);
    pages.clear();
}

// Pages for positions [len, len + n) of sequence seq: new pages from the
// pool, and a copy of the page holding position len when another sequence
// shares it (its rows below len stay valid in both).
static int reserve(aaedn_model* m, uint32_t seq, uint32_t n)
{
    auto& sq = m->seqs[seq];
    const uint32_t P = (uint32_t)m->page_size;
    if ((size_t)sq.len + n > m->cfg.max_seq)
        return set_error(AAEDN_ESTATE, "sequence %u full: %u + %u tokens > max_seq %u", seq, sq.len, n, m->cfg.max_seq);
    bool changed = false;
    if (n && sq.len % P != 0)
    {
        const size_t pi = sq.len / P;
        const int old = sq.pages[pi];
        if (m->page_ref[(size_t)old] > 1)
        {
            if (m->free_pages.empty())
                return set_error(AAEDN_ENOMEM, "KV page pool exhausted (%d pages)", m->n_pages);
            const int fresh = m->free_pages.back();
            m->free_pages.pop_back();
            const size_t pe = (size_t)m->cfg.n_kv_heads * P * m->cfg.head_dim; // floats per page per layer
            for (const DevLayer& L : m->layers)
            {
                AAEDN_CUDA_TRY(cudaMemcpyAsync(L.k + (size_t)fresh * pe, L.k + (size_t)old * pe, pe * 4,
                                               cudaMemcpyDeviceToDevice, m->stream));
                AAEDN_CUDA_TRY(cudaMemcpyAsync(L.v + (size_t)fresh * pe, L.v + (size_t)old * pe, pe * 4,
                                               cudaMemcpyDeviceToDevice, m->stream));
            }
            --m->page_ref[(size_t)old];
            m->page_ref[(size_t)fresh] = 1;
            sq.pages[pi] = fresh;
            changed = true;
        }
    }
    const size_t need = ((size_t)sq.len + n + P - 1) / P;
    while (sq.pages.size() < need)
    {
        if (m->free_pages.empty())
            return set_error(AAEDN_ENOMEM, "KV page pool exhausted (%d pages)", m->n_pages);
        const int pg = m->free_pages.back();
        m->free_pages.pop_back();
        m->page_ref[(size_t)pg] = 1;
        sq.pages.push_back(pg);
        changed = true;
    }
    return changed ? upload_pt(m, seq) : AAEDN_OK;
}

// The final RMSNorm, lm_head and greedy token of n rows of m->pf_hidden
// starting at row0, into b_logits / b_next rows [0, n).
static int lm_rows(aaedn_model* m, int row0, int n)
{
    cudaStream_t st = m->stream;
    const int D = (int)m->cfg.dim, V = (int)m->cfg.vocab;
    pf_rmsnorm_rows_kernel<<<n, 256, 0, st>>>(m->pf_hidden + (size_t)row0 * D, D, m->final_norm, m->cfg.eps,
                                               m->b_norm);
    AAEDN_LAUNCH_CHECK("pf_rmsnorm_rows_kernel");
    int parts;
    if (n <= LF_MAXM && D % 128 == 0)
    {
        // a few rows (a prefill's last token): stream the lm_head once
        parts = 2 * sm_count();
        lm_rows_few_kernel<<<parts, LF_WARPS * 32, (size_t)n * D * 4, st>>>(m->b_norm, n, D, m->lm_head, V,
                                                                           m->b_logits, (size_t)V, m->b_pval,
                                                                           m->b_pidx);
        AAEDN_LAUNCH_CHECK("lm_rows_few_kernel");
    }
    else
    {
        parts = (V + LR_BN - 1) / LR_BN;
        lm_rows_kernel<<<dim3(parts, (n + LR_BM - 1) / LR_BM), 256, lm_rows_smem_bytes(), st>>>(
            m->b_norm, n, D, m->lm_head, V, m->b_logits, (size_t)V, m->b_pval, m->b_pidx);
        AAEDN_LAUNCH_CHECK("lm_rows_kernel");
    }
    argmax_parts_kernel<<<(n + 7) / 8, 256, 0, st>>>(m->b_pval, m->b_pidx, parts, n, m->b_next);
    AAEDN_LAUNCH_CHECK("argmax_parts_kernel");
    return AAEDN_OK;
}

extern "C" int aaedn_model_create_batched(const aaedn_model_config* cfg, uint32_t max_seqs, uint64_t kv_tokens,
                                          aaedn_model** out)
{
    if (!cfg || !out)
        return set_error(AAEDN_EINVAL, "aaedn_model_create_batched: null argument");
    if (max_seqs == 0 || max_seqs > 256 || kv_tokens == 0 || kv_tokens > (1ull << 26))
        return set_error(AAEDN_EINVAL, "aaedn_model_create_batched: 1..256 sequences and 1..2^26 cached tokens");
    return create_impl(cfg, 0, 1, out, max_seqs, kv_tokens);
}

extern "C" int aaedn_seq_open(aaedn_model* m, uint32_t* seq)
{
    BATCHED_OK(m);
    if (!seq)
        return set_error(AAEDN_EINVAL, "aaedn_seq_open: null output");
    for (uint32_t i = 0; i < m->max_seqs; ++i)
        if (!m->seqs[i].open)
        {
            m->seqs[i] = aaedn_model::Seq{};
            m->seqs[i].open = true;
            *seq = i;
            return AAEDN_OK;
        }
    return set_error(AAEDN_ENOMEM, "all %u sequences are open", m->max_seqs);
}

extern "C" int aaedn_seq_fork(aaedn_model* m, uint32_t parent, uint32_t* child)
{
    BATCHED_OK(m);
    if (int rc = seq_ok(m, parent))
        return rc;
    uint32_t c = 0;
    if (int rc = aaedn_seq_open(m, &c))
        return rc;
    m->seqs[c].len = m->seqs[parent].len;
    m->seqs[c].pages = m->seqs[parent].pages;
    for (int pg : m->seqs[c].pages)
        ++m->page_ref[(size_t)pg];
    if (int rc = upload_pt(m, c))
        return rc;
    *child = c;
    return AAEDN_OK;
}

extern "C" int aaedn_seq_close(aaedn_model* m, uint32_t seq)
{
    BATCHED_OK(m);
    if (int rc = seq_ok(m, seq))
        return rc;
    // stream order: kernels still reading its pages were enqueued before
    // any later write that reuses them
    release_pages(m, m->seqs[seq].pages);
    m->seqs[seq].open = false;
    m->seqs[seq].len = 0;
    return AAEDN_OK;
}

extern "C" int aaedn_seq_len(aaedn_model* m, uint32_t seq, uint32_t* len)
{
    BATCHED_OK(m);
    if (int rc = seq_ok(m, seq))
        return rc;
    if (!len)
        return set_error(AAEDN_EINVAL, "aaedn_seq_len: null output");
    *len = m->seqs[seq].len;
    return AAEDN_OK;
}

extern "C" int aaedn_model_kv_pages(aaedn_model* m, uint32_t* total, uint32_t* free_pages)
{
    BATCHED_OK(m);
    if (total)
        *total = (uint32_t)m->n_pages;
    if (free_pages)
        *free_pages = (uint32_t)m->free_pages.size();
    return AAEDN_OK;
}

extern "C" int aaedn_seq_prefill(aaedn_model* m, uint32_t seq, const uint32_t* h_tokens, size_t n, float* h_logits,
                                 uint32_t* h_next)
{
    BATCHED_OK(m);
    if (int rc = seq_ok(m, seq))
        return rc;
    if (!h_tokens || n == 0)
        return set_error(AAEDN_EINVAL, "aaedn_seq_prefill: no tokens");
    for (size_t i = 0; i < n; ++i)
        if (h_tokens[i] >= m->cfg.vocab)
            return set_error(AAEDN_EINVAL, "token id %u >= vocab %u", h_tokens[i], m->cfg.vocab);
    if (int rc = reserve(m, seq, (uint32_t)n))
        return rc;
    // tokens into the model's prompt buffer (the staging is reused only
    // after the stream has drained)
    AAEDN_CUDA_TRY(cudaStreamSynchronize(m->stream));
    std::memcpy(m->pinned, h_tokens, n * 4);
    AAEDN_CUDA_TRY(cudaMemcpyAsync(m->prompt, m->pinned, n * 4, cudaMemcpyHostToDevice, m->stream));
    const uint32_t p0 = m->seqs[seq].len;
    const int* pt = m->seq_pt + (size_t)seq * m->pt_stride;
    size_t last = 0;
    for (size_t c0 = 0; c0 < n; c0 += (size_t)m->pf_rows)
    {
        const int nc = (int)std::min<size_t>((size_t)m->pf_rows, n - c0);
        if (int rc = prefill_chunk(m, m->prompt + c0, nc, RowMap{pt, p0 + (uint32_t)c0, nullptr, nullptr, 0}))
            return rc;
        last = (size_t)nc - 1;
    }
    if (int rc = lm_rows(m, (int)last, 1))
        return rc;
    if (h_logits)
        AAEDN_CUDA_TRY(cudaMemcpyAsync(h_logits, m->b_logits, (size_t)m->cfg.vocab * 4, cudaMemcpyDeviceToHost,
                                       m->stream));
    if (h_next)
        AAEDN_CUDA_TRY(cudaMemcpyAsync(h_next, m->b_next, 4, cudaMemcpyDeviceToHost, m->stream));
    AAEDN_CUDA_TRY(cudaStreamSynchronize(m->stream));
    m->seqs[seq].len += (uint32_t)n;
    return device_status(m);
}

extern "C" int aaedn_model_step_batch(aaedn_model* m, const uint32_t* h_seqs, const uint32_t* h_tokens, size_t n,
                                      float* h_logits, uint32_t* h_next)
{
    BATCHED_OK(m);
    if (!h_seqs || !h_tokens || n == 0 || n > m->max_seqs)
        return set_error(AAEDN_EINVAL, "aaedn_model_step_batch: 1..%u sequences", m->max_seqs);
    std::vector<uint8_t> seen(m->max_seqs, 0);
    for (size_t i = 0; i < n; ++i)
    {
        if (int rc = seq_ok(m, h_seqs[i]))
            return rc;
        if (seen[h_seqs[i]]++)
            return set_error(AAEDN_EINVAL, "sequence %u twice in one batch", h_seqs[i]);
        if (h_tokens[i] >= m->cfg.vocab)
            return set_error(AAEDN_EINVAL, "token id %u >= vocab %u", h_tokens[i], m->cfg.vocab);
    }
    for (size_t i = 0; i < n; ++i)
        if (int rc = reserve(m, h_seqs[i], 1))
            return rc;
    AAEDN_CUDA_TRY(cudaStreamSynchronize(m->stream)); // the staging may still feed an earlier copy
    int* stg = m->pinned_b;
    for (size_t i = 0; i < n; ++i)
    {
        stg[i] = (int)h_tokens[i];
        stg[m->max_seqs + i] = (int)m->seqs[h_seqs[i]].len;
        stg[2 * m->max_seqs + i] = (int)h_seqs[i];
    }
    AAEDN_CUDA_TRY(cudaMemcpyAsync(m->b_tokens, stg, n * 4, cudaMemcpyHostToDevice, m->stream));
    AAEDN_CUDA_TRY(cudaMemcpyAsync(m->b_pos, stg + m->max_seqs, n * 4, cudaMemcpyHostToDevice, m->stream));
    AAEDN_CUDA_TRY(cudaMemcpyAsync(m->b_seq, stg + 2 * m->max_seqs, n * 4, cudaMemcpyHostToDevice, m->stream));
    int rc = prefill_chunk(m, m->b_tokens, (int)n, RowMap{m->seq_pt, 0u, m->b_pos, m->b_seq, (int)m->pt_stride});
    if (!rc)
        rc = lm_rows(m, 0, (int)n);
    if (rc)
        return rc;
    if (h_logits)
        AAEDN_CUDA_TRY(cudaMemcpyAsync(h_logits, m->b_logits, n * m->cfg.vocab * 4, cudaMemcpyDeviceToHost,
                                       m->stream));
    if (h_next)
        AAEDN_CUDA_TRY(cudaMemcpyAsync(h_next, m->b_next, n * 4, cudaMemcpyDeviceToHost, m->stream));
    AAEDN_CUDA_TRY(cudaStreamSynchronize(m->stream));
    for (size_t i = 0; i < n; ++i)
        ++m->seqs[h_seqs[i]].len;
    return device_status(m);
}
