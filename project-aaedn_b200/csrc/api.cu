// api.cu — C ABI of the primitive kernels (dequant, fused_matmul, f32
// matmul, rmsnorm, rope_apply, attention) and the device helpers.
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "attention.cuh"
#include "gemm_tc.h"
#include "gemv_q4.cuh"

namespace aaedn_dev
{
std::atomic<uint64_t> g_launches{0};

// ---------------------------------------------------------------------------
// dequant_4bit: src/dequant.cpp:7-28. Thread i handles elements 8i..8i+7
// (4 bytes of codes); out = (float)code * scale is exact in fp32.
// ---------------------------------------------------------------------------
template <int SK>
__global__ void dequant_kernel(const uint8_t* __restrict__ data, const uint16_t* __restrict__ scales,
                               float* __restrict__ out, size_t n, int zero_all)
{
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    const size_t e0 = i * 8;
    if (e0 >= n)
        return;
    const size_t cnt = (n - e0) < 8 ? (n - e0) : 8;
    if (zero_all || scales[0] == 0) // src/dequant.cpp:9-14
    {
        for (size_t c = 0; c < cnt; ++c)
            out[e0 + c] = 0.0f;
        return;
    }
    const float sc = decode_scale<SK>(scales[e0 >> 5]); // 8 elements never straddle a block
    float v[8];
#pragma unroll
    for (int c = 0; c < 8; ++c)
    {
        if ((size_t)c < cnt)
        {
            const uint8_t byte = data[(e0 + c) >> 1];
            const uint32_t code = (c & 1) ? (byte >> 4) & 0x0F : byte & 0x0F;
            v[c] = (float)code * sc;
        }
    }
    if (cnt == 8 && (reinterpret_cast<uintptr_t>(out + e0) & 15) == 0)
    {
        reinterpret_cast<float4*>(out + e0)[0] = make_float4(v[0], v[1], v[2], v[3]);
        reinterpret_cast<float4*>(out + e0)[1] = make_float4(v[4], v[5], v[6], v[7]);
    }
    else
    {
        for (size_t c = 0; c < cnt; ++c)
            out[e0 + c] = v[c];
    }
}

// ---------------------------------------------------------------------------
// rmsnorm: src/rmsnorm.cpp:8-51, one CTA.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(1024) rmsnorm_kernel(const float* __restrict__ in, float* __restrict__ out,
                                                       const float* __restrict__ w, size_t n, float eps)
{
    __shared__ float scratch[64];
    float ss = 0.0f;
    for (size_t i = threadIdx.x; i < n; i += blockDim.x)
        ss = fmaf(in[i], in[i], ss);
    ss = block_sum(ss, scratch);
    const float rms = 1.0f / sqrtf(__fadd_rn(__fdiv_rn(ss, (float)n), eps));
    for (size_t i = threadIdx.x; i < n; i += blockDim.x)
        out[i] = __fmul_rn(__fmul_rn(in[i], rms), w[i]);
}

// ---------------------------------------------------------------------------
// rope_apply: src/rope.cpp:36-63
// ---------------------------------------------------------------------------
__global__ void rope_apply_kernel(float* __restrict__ q, float* __restrict__ k, size_t seq_len, size_t hd,
                                  const float* __restrict__ cos_t, const float* __restrict__ sin_t)
{
    const size_t half = hd / 2;
    const size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= seq_len * half)
        return;
    const size_t pos = idx / half, i = idx - pos * half;
    const float c = cos_t[pos * half + i], s = sin_t[pos * half + i];
    const size_t a = pos * hd + i, b = a + half;
    const float q0 = q[a], q1 = q[b];
    q[a] = __fsub_rn(__fmul_rn(c, q0), __fmul_rn(s, q1));
    q[b] = __fadd_rn(__fmul_rn(s, q0), __fmul_rn(c, q1));
    const float k0 = k[a], k1 = k[b];
    k[a] = __fsub_rn(__fmul_rn(c, k0), __fmul_rn(s, k1));
    k[b] = __fadd_rn(__fmul_rn(s, k0), __fmul_rn(c, k1));
}

// ---------------------------------------------------------------------------
// fp32 matmul (lm_head form): one warp per output element.
// ---------------------------------------------------------------------------
__global__ void f32_matmul_kernel(const float* __restrict__ in, const float* __restrict__ w, float* __restrict__ out,
                                  size_t M, size_t N, size_t K, size_t lda, size_t ldw, size_t ldc)
{
    const size_t gw = ((size_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (gw >= M * N)
        return;
    const size_t m = gw / N, n = gw - m * N;
    const float* x = in + m * lda;
    const float* wr = w + n * ldw;
    float acc = 0.0f;
    for (size_t k = lane; k < K; k += 32)
        acc = fmaf(x[k], wr[k], acc);
    acc = warp_sum(acc);
    if (lane == 0)
        out[m * ldc + n] = acc;
}

__global__ void zero_kernel(float* out, size_t n)
{
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n)
        out[i] = 0.0f;
}

// ---------------------------------------------------------------------------
// fused_matmul launcher: M rows in chunks of <= 8, K in chunks that fit in
// shared memory (first chunk stores, later chunks accumulate).
// ---------------------------------------------------------------------------
template <int NM, int SK>
static int gemv_dispatch(const GemvParams& p, int first_chunk, cudaStream_t st)
{
    const int full = (p.full_shape && p.scale_pairs) ? 1 : 0;
    auto kern = first_chunk ? (full ? gemv_q4_kernel<NM, PRO_PLAIN, EPI_STORE, SK, true>
                                    : gemv_q4_kernel<NM, PRO_PLAIN, EPI_STORE, SK, false>)
                            : (full ? gemv_q4_kernel<NM, PRO_PLAIN, EPI_ACCUM, SK, true>
                                    : gemv_q4_kernel<NM, PRO_PLAIN, EPI_ACCUM, SK, false>);
    // per device (the attribute is set on the current device only)
    static PerDeviceOnce attr_done[2][2];
    const int arc = attr_done[first_chunk][full].run([&]() -> int {
        AAEDN_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
        return AAEDN_OK;
    });
    if (arc)
        return arc;
    const int groups = (p.N + 15) / 16;
    const int grid = groups < sm_count() ? groups : sm_count();
    const size_t smem = gemv_smem_bytes(NM, p.kt1 - p.kt0);
    kern<<<grid, GEMV_WARPS * 32, smem, st>>>(p);
    AAEDN_LAUNCH_CHECK("gemv_q4_kernel");
    return AAEDN_OK;
}

template <int SK>
static int gemv_dispatch_m(int nm, const GemvParams& p, int first_chunk, cudaStream_t st)
{
    switch (nm)
    {
    case 1: return gemv_dispatch<1, SK>(p, first_chunk, st);
    case 2: return gemv_dispatch<2, SK>(p, first_chunk, st);
    case 3: return gemv_dispatch<3, SK>(p, first_chunk, st);
    case 4: return gemv_dispatch<4, SK>(p, first_chunk, st);
    case 5: return gemv_dispatch<5, SK>(p, first_chunk, st);
    case 6: return gemv_dispatch<6, SK>(p, first_chunk, st);
    case 7: return gemv_dispatch<7, SK>(p, first_chunk, st);
    default: return gemv_dispatch<8, SK>(p, first_chunk, st);
    }
}

} // namespace aaedn_dev

using namespace aaedn_dev;

// Rejects host pointers: the kernels need device-accessible memory.
static int check_dev(const void* p, const char* what)
{
    if (!p)
        return set_error(AAEDN_EINVAL, "%s is null", what);
    cudaPointerAttributes a;
    cudaError_t e = cudaPointerGetAttributes(&a, p);
    if (e != cudaSuccess)
    {
        cudaGetLastError();
        return set_error(AAEDN_EINVAL, "%s: cannot query pointer (%s)", what, cudaGetErrorString(e));
    }
    if (a.type != cudaMemoryTypeDevice && a.type != cudaMemoryTypeManaged)
        return set_error(AAEDN_EINVAL, "%s is not device memory", what);
    return AAEDN_OK;
}

#define CHECK_DEV(p)                                                                                          \
    do                                                                                                        \
    {                                                                                                         \
        int _rc = check_dev((p), #p);                                                                         \
        if (_rc)                                                                                              \
            return _rc;                                                                                       \
    } while (0)

extern "C" uint64_t aaedn_kernel_launches(void) { return g_launches.load(); }

extern "C" int aaedn_dev_alloc(void** d_ptr, size_t bytes)
{
    if (!d_ptr)
        return set_error(AAEDN_EINVAL, "aaedn_dev_alloc: null out pointer");
    *d_ptr = nullptr;
    cudaError_t e = cudaMalloc(d_ptr, bytes ? bytes : 1);
    if (e != cudaSuccess)
        return set_error(e == cudaErrorMemoryAllocation ? AAEDN_ENOMEM : AAEDN_ECUDA, "cudaMalloc(%zu): %s", bytes,
                         cudaGetErrorString(e));
    return AAEDN_OK;
}

extern "C" int aaedn_dev_free(void* d_ptr)
{
    AAEDN_CUDA_TRY(cudaFree(d_ptr));
    return AAEDN_OK;
}

extern "C" int aaedn_memcpy_h2d(void* d_dst, const void* h_src, size_t bytes, void* stream)
{
    AAEDN_CUDA_TRY(cudaMemcpyAsync(d_dst, h_src, bytes, cudaMemcpyHostToDevice, as_stream(stream)));
    return AAEDN_OK;
}

extern "C" int aaedn_memcpy_d2h(void* h_dst, const void* d_src, size_t bytes, void* stream)
{
    AAEDN_CUDA_TRY(cudaMemcpyAsync(h_dst, d_src, bytes, cudaMemcpyDeviceToHost, as_stream(stream)));
    return AAEDN_OK;
}

extern "C" int aaedn_stream_sync(void* stream)
{
    AAEDN_CUDA_TRY(cudaStreamSynchronize(as_stream(stream)));
    return AAEDN_OK;
}

extern "C" int aaedn_device_sync(void)
{
    AAEDN_CUDA_TRY(cudaDeviceSynchronize());
    return tc_api_err_check();
}

extern "C" int aaedn_cu_dequant_4bit(const uint8_t* d_data, const uint16_t* d_scales, float* d_out, size_t n,
                                     int scale_kind, void* stream)
{
    if (n == 0)
        return AAEDN_OK;
    CHECK_DEV(d_out);
    const int zero_all = (!d_data || !d_scales) ? 1 : 0; // src/dequant.cpp:9
    if (!zero_all)
    {
        CHECK_DEV(d_data);
        CHECK_DEV(d_scales);
    }
    const uint16_t* sp = zero_all ? nullptr : d_scales;
    const size_t threads = (n + 7) / 8;
    const unsigned grid = (unsigned)((threads + 255) / 256);
    if (zero_all)
    {
        zero_kernel<<<(unsigned)((n + 255) / 256), 256, 0, as_stream(stream)>>>(d_out, n);
        AAEDN_LAUNCH_CHECK("zero_kernel");
        return AAEDN_OK;
    }
    if (scale_kind == AAEDN_SCALE_F16)
        dequant_kernel<AAEDN_SCALE_F16><<<grid, 256, 0, as_stream(stream)>>>(d_data, sp, d_out, n, 0);
    else if (scale_kind == AAEDN_SCALE_U16INT)
        dequant_kernel<AAEDN_SCALE_U16INT><<<grid, 256, 0, as_stream(stream)>>>(d_data, sp, d_out, n, 0);
    else
        return set_error(AAEDN_EINVAL, "aaedn_cu_dequant_4bit: bad scale_kind %d", scale_kind);
    AAEDN_LAUNCH_CHECK("dequant_kernel");
    return AAEDN_OK;
}

extern "C" int aaedn_cu_fused_matmul(const float* d_in, const uint8_t* d_w, const uint16_t* d_scales, float* d_out,
                                     size_t M, size_t N, size_t K, size_t lda, size_t ldb, size_t ldc, int scale_kind,
                                     void* stream)
{
    if (M == 0 || N == 0 || K == 0) // src/fused_matmul.cpp:76-77
        return AAEDN_OK;
    if ((K & 31) || (ldb & 31) || ldb < K || lda < K || ldc < N)
        return set_error(AAEDN_EINVAL, "aaedn_cu_fused_matmul: K and ldb must be multiples of 32 with ldb>=K, "
                                       "lda>=K, ldc>=N (K=%zu ldb=%zu lda=%zu ldc=%zu N=%zu)",
                         K, ldb, lda, ldc, N);
    if (N > (size_t)INT32_MAX || K > (size_t)INT32_MAX)
        return set_error(AAEDN_EINVAL, "aaedn_cu_fused_matmul: N/K too large");
    if (scale_kind != AAEDN_SCALE_F16 && scale_kind != AAEDN_SCALE_U16INT)
        return set_error(AAEDN_EINVAL, "aaedn_cu_fused_matmul: bad scale_kind %d", scale_kind);
    CHECK_DEV(d_in);
    CHECK_DEV(d_w);
    CHECK_DEV(d_scales);
    CHECK_DEV(d_out);
    if ((reinterpret_cast<uintptr_t>(d_w) & 15) || ((ldb / 2) & 15))
        return set_error(AAEDN_EINVAL, "aaedn_cu_fused_matmul: weights must be 16-byte aligned rows");
    cudaStream_t st = as_stream(stream);
    if (M > 8 && scale_kind == AAEDN_SCALE_F16 && (K % 64) == 0 && M <= (size_t)INT32_MAX)
    {
        // many rows: the tensor-core GEMM (each weight read once per 128 x
        // up-to-128 tile instead of once per 8 rows)
        TcGemmArgs a{};
        a.x = d_in;
        a.lda = lda;
        a.M = (int)M;
        a.N = (int)N;
        a.K = (int)K;
        a.w = d_w;
        a.s = d_scales;
        a.ldb = ldb;
        a.w_layout = TC_W_ROWMAJOR;
        a.out = d_out;
        a.ldc = ldc;
        a.err = tc_api_err_word();
        if (!a.err)
            return set_error(AAEDN_ECUDA, "aaedn_cu_fused_matmul: error word allocation failed");
        a.workspace_bytes = tc_gemm_workspace_bytes(a.M, a.N, a.K);
        AAEDN_CUDA_TRY(cudaMallocAsync(&a.workspace, a.workspace_bytes, st));
        const int rc = tc_gemm(a, st);
        AAEDN_CUDA_TRY(cudaFreeAsync(a.workspace, st));
        return rc;
    }
    const int ntile_total = (int)((K + 127) / 128);
    for (size_t m0 = 0; m0 < M; m0 += 8)
    {
        const int nm = (int)((M - m0) < 8 ? (M - m0) : 8);
        // tiles per chunk so that ring + activation fragments fit in 200 KB
        const size_t fixed = gemv_smem_bytes(nm, 0);
        const int max_tiles = (int)((200 * 1024 - fixed) / ((size_t)nm * (GEMV_FRAG_TILE_BYTES + 16)));
        for (int kt0 = 0; kt0 < ntile_total; kt0 += max_tiles)
        {
            GemvParams p{};
            p.w = d_w;
            p.s = d_scales;
            p.ldb = ldb;
            p.N = (int)N;
            p.K = (int)K;
            p.kt0 = kt0;
            p.kt1 = kt0 + max_tiles < ntile_total ? kt0 + max_tiles : ntile_total;
            p.x = d_in + m0 * lda;
            p.lda = lda;
            p.y = d_out + m0 * ldc;
            p.ldc = ldc;
            p.scale_pairs = ((ldb >> 5) & 1) == 0 && (reinterpret_cast<uintptr_t>(d_scales) & 3) == 0;
            p.full_shape = (N % 16) == 0 && (K % 128) == 0;
            int rc = scale_kind == AAEDN_SCALE_F16 ? gemv_dispatch_m<AAEDN_SCALE_F16>(nm, p, kt0 == 0, st)
                                                   : gemv_dispatch_m<AAEDN_SCALE_U16INT>(nm, p, kt0 == 0, st);
            if (rc)
                return rc;
        }
    }
    return AAEDN_OK;
}

extern "C" int aaedn_cu_f32_matmul(const float* d_in, const float* d_w, float* d_out, size_t M, size_t N, size_t K,
                                   size_t lda, size_t ldw, size_t ldc, void* stream)
{
    if (M == 0 || N == 0)
        return AAEDN_OK;
    CHECK_DEV(d_in);
    CHECK_DEV(d_w);
    CHECK_DEV(d_out);
    const size_t warps = M * N;
    const unsigned grid = (unsigned)((warps * 32 + 255) / 256);
    f32_matmul_kernel<<<grid, 256, 0, as_stream(stream)>>>(d_in, d_w, d_out, M, N, K, lda, ldw, ldc);
    AAEDN_LAUNCH_CHECK("f32_matmul_kernel");
    return AAEDN_OK;
}

extern "C" int aaedn_cu_rmsnorm(const float* d_in, float* d_out, const float* d_w, size_t n, float eps, void* stream)
{
    if (n == 0)
        return AAEDN_OK;
    CHECK_DEV(d_in);
    CHECK_DEV(d_out);
    CHECK_DEV(d_w);
    rmsnorm_kernel<<<1, 1024, 0, as_stream(stream)>>>(d_in, d_out, d_w, n, eps);
    AAEDN_LAUNCH_CHECK("rmsnorm_kernel");
    return AAEDN_OK;
}

extern "C" int aaedn_cu_rope_apply(float* d_q, float* d_k, size_t seq_len, size_t head_dim, const float* d_cos,
                                   const float* d_sin, void* stream)
{
    if (!d_cos || !d_sin) // src/rope.cpp:38-39
        return AAEDN_OK;
    if (seq_len == 0 || head_dim < 2)
        return AAEDN_OK;
    CHECK_DEV(d_q);
    CHECK_DEV(d_k);
    CHECK_DEV(d_cos);
    CHECK_DEV(d_sin);
    const size_t work = seq_len * (head_dim / 2);
    rope_apply_kernel<<<(unsigned)((work + 255) / 256), 256, 0, as_stream(stream)>>>(d_q, d_k, seq_len, head_dim,
                                                                                     d_cos, d_sin);
    AAEDN_LAUNCH_CHECK("rope_apply_kernel");
    return AAEDN_OK;
}

// the attention kernels' shared-memory attribute, set once per device
static PerDeviceOnce g_attn_api_attrs;

extern "C" int aaedn_cu_attention(const float* d_q, const float* d_k, const float* d_v, const uint32_t* h_segments,
                                  size_t num_segments, float* d_out, size_t n_heads, size_t head_dim, float scale,
                                  void* stream)
{
    if (n_heads == 0 || head_dim == 0)
        return AAEDN_OK;
    CHECK_DEV(d_out);
    cudaStream_t st = as_stream(stream);
    size_t total = 0;
    if (h_segments)
        for (size_t i = 0; i < num_segments; ++i)
            total += h_segments[2 * i + 1];
    if (!d_q || !d_k || !d_v || !h_segments || total == 0) // src/attention.cpp:13-18
    {
        const size_t n = n_heads * head_dim;
        zero_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(d_out, n);
        AAEDN_LAUNCH_CHECK("zero_kernel");
        return AAEDN_OK;
    }
    if (num_segments > (size_t)ATTN_MAX_SEG || head_dim > (size_t)ATTN_MAX_HD || (head_dim & 3) ||
        total > (size_t)INT32_MAX)
        return set_error(AAEDN_EINVAL, "aaedn_cu_attention: at most %d segments and head_dim a multiple of 4 <= %d",
                         ATTN_MAX_SEG, ATTN_MAX_HD);
    if ((reinterpret_cast<uintptr_t>(d_q) | reinterpret_cast<uintptr_t>(d_k) | reinterpret_cast<uintptr_t>(d_v)) & 15)
        return set_error(AAEDN_EINVAL, "aaedn_cu_attention: q/k/v must be 16-byte aligned");
    CHECK_DEV(d_q);
    CHECK_DEV(d_k);
    CHECK_DEV(d_v);
    AttnParams p{};
    p.q = d_q;
    p.k = d_k;
    p.v = d_v;
    p.out = d_out;
    p.n_heads = (int)n_heads;
    p.n_kv = (int)n_heads;
    p.head_dim = (int)head_dim;
    p.scale = scale;
    p.len_static = (int)total;
    p.max_len = (int)total;
    int S = (int)((2 * 148 + n_heads - 1) / n_heads);
    if (S > (int)((total + 7) / 8))
        S = (int)((total + 7) / 8);
    if (S < 1)
        S = 1;
    if (S > 256)
        S = 256;
    p.S = S;
    p.max_tok = (int)((total + S - 1) / S);
    const size_t smem = attn_smem_bytes(1, (int)head_dim, p.max_tok);
    if (smem > 200 * 1024)
        return set_error(AAEDN_EINVAL, "aaedn_cu_attention: too many tokens per split");
    p.nseg = (int)num_segments;
    uint32_t off = 0;
    for (size_t i = 0; i < num_segments; ++i)
    {
        p.seg_start[i] = h_segments[2 * i];
        p.seg_off[i] = off;
        off += h_segments[2 * i + 1];
    }
    p.seg_off[num_segments] = off;
    // scratch: partials + counters (zeroed) for this call
    float* part = nullptr;
    unsigned* counters = nullptr;
    const size_t part_bytes = n_heads * (size_t)S * (head_dim + 2) * sizeof(float);
    AAEDN_CUDA_TRY(cudaMallocAsync(reinterpret_cast<void**>(&part), part_bytes + n_heads * sizeof(unsigned), st));
    counters = reinterpret_cast<unsigned*>(reinterpret_cast<uint8_t*>(part) + part_bytes);
    AAEDN_CUDA_TRY(cudaMemsetAsync(counters, 0, n_heads * sizeof(unsigned), st));
    p.part = part;
    p.counters = counters;
    int arc = g_attn_api_attrs.run([]() { return attn_set_attrs_g<0, 1>(); });
    if (arc)
    {
        cudaFreeAsync(part, st);
        return arc;
    }
    int lrc = attn_launch<0>(p, dim3((unsigned)n_heads, (unsigned)S), smem, st);
    AAEDN_CUDA_TRY(cudaFreeAsync(part, st));
    if (lrc)
        return lrc;
    return AAEDN_OK;
}

// ---------------------------------------------------------------------------
// Attention for callers that cannot allocate: the scratch is a fixed array in
// device global memory, resolved to a device address once per device.
// ---------------------------------------------------------------------------
namespace
{
constexpr size_t NOALLOC_COUNTER_BYTES = 4096; // split counters of up to 1024 heads
static __device__ __align__(256) uint8_t g_attn_noalloc_scratch[AAEDN_ATTN_NOALLOC_SCRATCH_BYTES];
std::mutex g_noalloc_mu;
uint8_t* g_noalloc_base[64] = {}; // device address of the array, per device

int noalloc_scratch(uint8_t** out)
{
    int dev = 0;
    AAEDN_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64)
        return set_error(AAEDN_EUNSUPPORTED, "aaedn_cu_attention_noalloc: device ordinal %d >= 64", dev);
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (!g_noalloc_base[dev])
    {
        // host code only sees a stand-in for the array: ask the runtime for
        // its address on the current device
        void* p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_attn_noalloc_scratch);
        if (e != cudaSuccess || !p)
            return set_error(AAEDN_ECUDA, "aaedn_cu_attention_noalloc: cudaGetSymbolAddress failed: %s",
                             cudaGetErrorString(e));
        g_noalloc_base[dev] = static_cast<uint8_t*>(p);
    }
    *out = g_noalloc_base[dev];
    return AAEDN_OK;
}
} // namespace

extern "C" int aaedn_cu_attention_noalloc(const float* d_q, const float* d_k, const float* d_v,
                                          const uint32_t* h_segments, size_t num_segments, float* d_out,
                                          size_t n_heads, size_t head_dim, float scale, void* stream)
{
    if (n_heads == 0 || head_dim == 0)
        return AAEDN_OK;
    CHECK_DEV(d_out);
    cudaStream_t st = as_stream(stream);
    size_t total = 0;
    if (h_segments)
        for (size_t i = 0; i < num_segments; ++i)
            total += h_segments[2 * i + 1];
    if (!d_q || !d_k || !d_v || !h_segments || total == 0) // src/attention.cpp:13-18
    {
        const size_t n = n_heads * head_dim;
        zero_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(d_out, n);
        AAEDN_LAUNCH_CHECK("zero_kernel");
        return AAEDN_OK;
    }
    if (num_segments > (size_t)ATTN_MAX_SEG || head_dim > (size_t)ATTN_MAX_HD || (head_dim & 3) ||
        total > (size_t)INT32_MAX)
        return set_error(AAEDN_EINVAL,
                         "aaedn_cu_attention_noalloc: at most %d segments and head_dim a multiple of 4 <= %d",
                         ATTN_MAX_SEG, ATTN_MAX_HD);
    const size_t part_cap = AAEDN_ATTN_NOALLOC_SCRATCH_BYTES - NOALLOC_COUNTER_BYTES;
    const size_t per_split = n_heads * (head_dim + 2) * sizeof(float);
    if (n_heads * sizeof(unsigned) > NOALLOC_COUNTER_BYTES || per_split > part_cap)
        return set_error(AAEDN_EINVAL,
                         "aaedn_cu_attention_noalloc: %zu heads x head_dim %zu need more than the %u-byte "
                         "scratch (at most 1024 heads and n_heads*(head_dim+2)*4 <= %zu bytes)",
                         n_heads, head_dim, AAEDN_ATTN_NOALLOC_SCRATCH_BYTES, part_cap);
    if ((reinterpret_cast<uintptr_t>(d_q) | reinterpret_cast<uintptr_t>(d_k) | reinterpret_cast<uintptr_t>(d_v)) & 15)
        return set_error(AAEDN_EINVAL, "aaedn_cu_attention_noalloc: q/k/v must be 16-byte aligned");
    CHECK_DEV(d_q);
    CHECK_DEV(d_k);
    CHECK_DEV(d_v);
    uint8_t* base = nullptr;
    int rc = noalloc_scratch(&base);
    if (rc)
        return rc;
    AttnParams p{};
    p.q = d_q;
    p.k = d_k;
    p.v = d_v;
    p.out = d_out;
    p.n_heads = (int)n_heads;
    p.n_kv = (int)n_heads;
    p.head_dim = (int)head_dim;
    p.scale = scale;
    p.len_static = (int)total;
    p.max_len = (int)total;
    // the split count of aaedn_cu_attention, capped by the scratch
    int S = (int)((2 * 148 + n_heads - 1) / n_heads);
    if (S > (int)((total + 7) / 8))
        S = (int)((total + 7) / 8);
    if (S > (int)(part_cap / per_split))
        S = (int)(part_cap / per_split);
    if (S < 1)
        S = 1;
    if (S > 256)
        S = 256;
    p.S = S;
    p.max_tok = (int)((total + S - 1) / S);
    const size_t smem = attn_smem_bytes(1, (int)head_dim, p.max_tok);
    if (smem > 200 * 1024)
        return set_error(AAEDN_EINVAL, "aaedn_cu_attention_noalloc: too many tokens per split");
    p.nseg = (int)num_segments;
    uint32_t off = 0;
    for (size_t i = 0; i < num_segments; ++i)
    {
        p.seg_start[i] = h_segments[2 * i];
        p.seg_off[i] = off;
        off += h_segments[2 * i + 1];
    }
    p.seg_off[num_segments] = off;
    p.counters = reinterpret_cast<unsigned*>(base);
    p.part = reinterpret_cast<float*>(base + NOALLOC_COUNTER_BYTES);
    // the array keeps whatever the last call left: the split counters must
    // start at zero (the partials are written before they are read)
    AAEDN_CUDA_TRY(cudaMemsetAsync(p.counters, 0, n_heads * sizeof(unsigned), st));
    const int arc = g_attn_api_attrs.run([]() { return attn_set_attrs_g<0, 1>(); });
    if (arc)
        return arc;
    return attn_launch<0>(p, dim3((unsigned)n_heads, (unsigned)S), smem, st);
}
