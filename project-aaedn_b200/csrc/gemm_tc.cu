// gemm_tc.cu — host side of the tcgen05 block-quantized GEMM (gemm_tc.cuh):
// the activation split, the TMA tensor map, tile / split-K selection and
// the deterministic split-K reduction.
#include <cudaTypedefs.h> // PFN_cuTensorMapEncodeTiled

#include <algorithm>
#include <mutex>

#include "gemm_tc.h"
#include "gemm_tc.cuh"

namespace aaedn_dev
{

namespace
{

PFN_cuTensorMapEncodeTiled_v12000 encode_fn()
{
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, []() {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

struct TcShape
{
    int bn, stages;
};

TcShape tc_shape(int M)
{
    // as many stages as shared memory holds
    if (M <= 32)
        return {32, 5};
    if (M <= 64)
        return {64, 4};
    return {128, 2};
}

template <int BN, int STAGES, int EPI>
int tc_launch(const TcGemmParams& p, const CUtensorMap& map, dim3 grid, cudaStream_t st)
{
    static PerDeviceOnce attr;
    constexpr size_t smem = TcSmem<BN, STAGES>::BYTES;
    int rc = attr.run([]() -> int {
        AAEDN_CUDA_TRY(cudaFuncSetAttribute(q4_gemm_tc_kernel<BN, STAGES, EPI>,
                                            cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        return AAEDN_OK;
    });
    if (rc)
        return rc;
    q4_gemm_tc_kernel<BN, STAGES, EPI><<<grid, TC_THREADS, smem, st>>>(p, map);
    AAEDN_LAUNCH_CHECK("q4_gemm_tc_kernel");
    return AAEDN_OK;
}

template <int EPI>
int tc_launch_bn(int bn, const TcGemmParams& p, const CUtensorMap& map, dim3 grid, cudaStream_t st)
{
    switch (bn)
    {
    case 32: return tc_launch<32, 5, EPI>(p, map, grid, st);
    case 64: return tc_launch<64, 4, EPI>(p, map, grid, st);
    default: return tc_launch<128, 2, EPI>(p, map, grid, st);
    }
}

// The split count: enough CTAs for every SM when the tile grid alone is
// small, at least 4 stages of K per CTA.
int tc_splits(int tiles, int nkb)
{
    int s = std::max(1, sm_count() / std::max(1, tiles));
    s = std::min(s, std::max(1, nkb / 4));
    const int per = (nkb + s - 1) / s;
    return (nkb + per - 1) / per;
}

} // namespace

int tc_m_pad(int M)
{
    const int bn = tc_shape(M).bn;
    return (M + bn - 1) / bn * bn;
}

void* tc_gemm_parts(void* workspace) { return workspace; }

int tc_split(const float* x, size_t lda, int M, int K, void* workspace, cudaStream_t st)
{
    const int M_pad = tc_m_pad(M);
    const size_t work = (size_t)M_pad * (K / 8);
    tc_split_kernel<<<(unsigned)((work + 255) / 256), 256, 0, st>>>(
        x, lda, M, M_pad, K, reinterpret_cast<__nv_bfloat16*>(tc_gemm_parts(workspace)));
    AAEDN_LAUNCH_CHECK("tc_split_kernel");
    return AAEDN_OK;
}

size_t tc_gemm_workspace_bytes(int M, int N, int K)
{
    const TcShape sh = tc_shape(M);
    const size_t M_pad = (size_t)(M + sh.bn - 1) / sh.bn * sh.bn;
    const int tiles = ((N + TC_BM - 1) / TC_BM) * (int)(M_pad / sh.bn);
    const int splits = tc_splits(tiles, K / TC_BK);
    size_t b = (TC_XP * M_pad * (size_t)K * 2 + 1023) / 1024 * 1024;
    if (splits > 1)
        b += (size_t)splits * M * N * 4;
    return b + 256;
}

int tc_gemm(const TcGemmArgs& a, cudaStream_t st)
{
    if (a.M <= 0 || a.N <= 0 || a.K <= 0)
        return AAEDN_OK;
    if (a.K % TC_BK)
        return set_error(AAEDN_EINVAL, "tensor-core GEMM: K = %d is not a multiple of %d", a.K, TC_BK);
    if (a.w_layout == TC_W_TILED && (a.K % 128 || a.N % 16))
        return set_error(AAEDN_EINVAL, "tensor-core GEMM: the tile-major layout needs K %% 128 == 0, N %% 16 == 0");
    if (!a.workspace || a.workspace_bytes < tc_gemm_workspace_bytes(a.M, a.N, a.K))
        return set_error(AAEDN_EINVAL, "tensor-core GEMM: workspace of %zu bytes, need %zu", a.workspace_bytes,
                         tc_gemm_workspace_bytes(a.M, a.N, a.K));
    auto encode = encode_fn();
    if (!encode)
        return set_error(AAEDN_ECUDA, "tensor-core GEMM: cuTensorMapEncodeTiled is not available");
    const TcShape sh = tc_shape(a.M);
    const int M_pad = (a.M + sh.bn - 1) / sh.bn * sh.bn;
    const int gx = (a.N + TC_BM - 1) / TC_BM, gy = M_pad / sh.bn;
    const int nkb = a.K / TC_BK;
    // split-K when the tile grid leaves SMs idle (the reduction then applies
    // the epilogue, the paired ones included)
    const int splits = tc_splits(gx * gy, nkb);
    const int kb_per = (nkb + splits - 1) / splits;
    uint8_t* ws = static_cast<uint8_t*>(a.workspace);
    __nv_bfloat16* parts = reinterpret_cast<__nv_bfloat16*>(ws);
    size_t off = (TC_XP * (size_t)M_pad * a.K * 2 + 1023) / 1024 * 1024;
    float* partial = nullptr;
    if (splits > 1)
    {
        partial = reinterpret_cast<float*>(ws + off);
        off += (size_t)splits * a.M * a.N * 4;
    }
    // the activation parts (unless the caller wrote them into the workspace)
    if (a.x)
    {
        const size_t work = (size_t)M_pad * (a.K / 8);
        tc_split_kernel<<<(unsigned)((work + 255) / 256), 256, 0, st>>>(a.x, a.lda, a.M, M_pad, a.K, parts);
        AAEDN_LAUNCH_CHECK("tc_split_kernel");
    }
    CUtensorMap map;
    const cuuint64_t dims[2] = {(cuuint64_t)a.K, (cuuint64_t)TC_XP * M_pad};
    const cuuint64_t strides[1] = {(cuuint64_t)a.K * 2};
    const cuuint32_t box[2] = {(cuuint32_t)TC_BK, (cuuint32_t)sh.bn};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult cr = encode(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, parts, dims, strides, box, estr,
                               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (cr != CUDA_SUCCESS)
        return set_error(AAEDN_ECUDA, "tensor-core GEMM: cuTensorMapEncodeTiled failed (%d)", (int)cr);
    TcGemmParams p{};
    p.w = a.w;
    p.s = a.s;
    p.ldb = a.ldb;
    p.w_layout = a.w_layout;
    p.N = a.N;
    p.K = a.K;
    p.M = a.M;
    p.k_per_split = kb_per * TC_BK;
    p.err = a.err;
    p.e = a.e;
    if (splits > 1)
    {
        p.out = partial;
        p.ldc = (size_t)a.N;
        p.split_stride = (size_t)a.M * a.N;
    }
    else
    {
        p.out = a.out;
        p.ldc = a.ldc;
        p.split_stride = 0;
    }
    const dim3 grid((unsigned)gx, (unsigned)gy, (unsigned)splits);
    int rc;
    const int epi = splits > 1 ? TC_EPI_STORE : a.epi; // split-K: partials, the epilogue in the reduction
    switch (epi)
    {
    case TC_EPI_RESID: rc = tc_launch_bn<TC_EPI_RESID>(sh.bn, p, map, grid, st); break;
    case TC_EPI_QKV: rc = tc_launch_bn<TC_EPI_QKV>(sh.bn, p, map, grid, st); break;
    case TC_EPI_SWIGLU: rc = tc_launch_bn<TC_EPI_SWIGLU>(sh.bn, p, map, grid, st); break;
    default: rc = tc_launch_bn<TC_EPI_STORE>(sh.bn, p, map, grid, st); break;
    }
    if (rc)
        return rc;
    if (splits > 1 && (a.epi == TC_EPI_QKV || a.epi == TC_EPI_SWIGLU))
    {
        const size_t n = (size_t)a.M * (a.N / 16) * 8;
        if (a.epi == TC_EPI_QKV)
            tc_splitk_pair_kernel<TC_EPI_QKV><<<(unsigned)((n + 255) / 256), 256, 0, st>>>(
                partial, splits, (size_t)a.M * a.N, a.M, a.N, a.e);
        else
            tc_splitk_pair_kernel<TC_EPI_SWIGLU><<<(unsigned)((n + 255) / 256), 256, 0, st>>>(
                partial, splits, (size_t)a.M * a.N, a.M, a.N, a.e);
        AAEDN_LAUNCH_CHECK("tc_splitk_pair_kernel");
    }
    else if (splits > 1)
    {
        const size_t n = (size_t)a.M * a.N;
        tc_splitk_reduce_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(
            partial, splits, (size_t)a.M * a.N, a.M, a.N, a.out, a.ldc, a.epi == TC_EPI_RESID ? 1 : 0);
        AAEDN_LAUNCH_CHECK("tc_splitk_reduce_kernel");
    }
    return AAEDN_OK;
}

namespace
{
std::mutex g_err_mu;
unsigned* g_err_word[64] = {};
} // namespace

unsigned* tc_api_err_word()
{
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64)
        return nullptr;
    std::lock_guard<std::mutex> lk(g_err_mu);
    if (!g_err_word[dev])
    {
        unsigned* w = nullptr;
        if (cudaMalloc(reinterpret_cast<void**>(&w), 4) != cudaSuccess || cudaMemset(w, 0, 4) != cudaSuccess)
            return nullptr;
        g_err_word[dev] = w;
    }
    return g_err_word[dev];
}

int tc_api_err_check()
{
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64)
        return AAEDN_OK;
    unsigned* w = nullptr;
    {
        std::lock_guard<std::mutex> lk(g_err_mu);
        w = g_err_word[dev];
    }
    if (!w)
        return AAEDN_OK;
    unsigned h = 0;
    AAEDN_CUDA_TRY(cudaMemcpy(&h, w, 4, cudaMemcpyDeviceToHost));
    if (h == 0)
        return AAEDN_OK;
    AAEDN_CUDA_TRY(cudaMemset(w, 0, 4));
    return set_error(AAEDN_ETIMEOUT, "a bounded wait of a tensor-core GEMM ran out (its output is undefined)");
}

} // namespace aaedn_dev
