// gemm_tc.h — host interface of the tcgen05 block-quantized GEMM
// (gemm_tc.cuh / gemm_tc.cu): out[m][n] = sum_k x[m][k] * code(n, k) *
// scale(n, k / 32) for M activation rows, fp32 in and out, fp32-accurate.
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

namespace aaedn_dev
{

// Order of the K elements inside every group of 8 in the GEMM's operands
// (and so in the activation parts written for it): k = 4 h + j sits at
// position 2 j + h, the order in which a 32-bit word's 8 codes come out as
// bf16 pairs (code j, code j + 4). The MMA sums over k, so any order shared
// by both operands gives the same product.
__host__ __device__ constexpr int tc_kpos(int k) { return (k & ~7) | ((k & 3) << 1) | ((k >> 2) & 1); }

// Weight layouts the GEMM reads.
enum
{
    TC_W_ROWMAJOR = 0, // [N][ldb] codes (ldb / 2 bytes per row), scales [N][ldb / 32]
    TC_W_TILED = 1,    // the decode GEMV's tile-major repacking (gemv_tiled.cuh)
};

// Epilogues of the GEMM (applied to D[n][m] = the product for weight row n
// and activation row m).
enum
{
    TC_EPI_STORE = 0,  // out[m * ldc + n] = D
    TC_EPI_RESID = 1,  // out[m * ldc + n] += D (the residual stream)
    TC_EPI_QKV = 2,    // RoPE on q and k rows, k/v appended to the paged cache at position pos0 + m
    TC_EPI_SWIGLU = 3, // act[m * ld_act + 8 j + r] = silu(D[16 j + r]) * D[16 j + 8 + r], r < 8
};

// What the model's epilogues need. QKV rows are in the model's device order:
// within every 16-row group, rows r and r + 8 are a RoPE pair (i, i + hd/2)
// of q or k, or dims (d, d + 8) of v; gate and up rows alternate in 8-row
// chunks.
struct TcEpi
{
    float* qrows; // [M][ldq]: q of every activation row, logical head order
    size_t ldq;
    float* k_layer; // paged cache [page][n_kv][page_size][head_dim]
    float* v_layer;
    const int* page_table; // one sequence's, or (row_seq) the base of [sequences][pt_stride]
    int page_size, n_kv, head_dim, q_rows, kv_rows, pos0;
    // activation rows of different sequences (batched decode): row m is at
    // position row_pos[m] of sequence row_seq[m], whose page table starts at
    // page_table + row_seq[m] * pt_stride; null: row m at pos0 + m of the one
    // sequence of page_table
    const int* row_pos;
    const int* row_seq;
    int pt_stride;
    const float* rope_cos; // [max_seq][head_dim / 2]
    const float* rope_sin;
    float* act; // [M][ld_act]
    size_t ld_act;
};

struct TcGemmArgs
{
    const float* x;   // [M][lda] fp32; null: the parts are already in the workspace (tc_gemm_parts)
    size_t lda;
    int M, N, K;      // K a multiple of 64
    const uint8_t* w; // codes: row-major [N][ldb / 2] bytes, or the tile-major repacking
    const uint16_t* s; // row-major scales [N][ldb / 32] (unused by the tile-major layout)
    size_t ldb;
    int w_layout;     // TC_W_ROWMAJOR or TC_W_TILED
    float* out;       // [M][ldc]
    size_t ldc;
    void* workspace;  // device memory of tc_gemm_workspace_bytes(M, N, K)
    size_t workspace_bytes;
    unsigned* err;    // device word set to 1 when a bounded wait ran out (may be null)
    int epi;          // TC_EPI_*
    TcEpi e;
};

size_t tc_gemm_workspace_bytes(int M, int N, int K);
// Where the workspace holds the activation parts ([3][tc_m_pad(M)][K] bf16)
// and the padded row count the GEMM reads.
int tc_m_pad(int M);
void* tc_gemm_parts(void* workspace);
// Writes the three bf16 parts of x ([M][lda] fp32, first K columns) into the
// workspace for a following tc_gemm with x = null.
int tc_split(const float* x, size_t lda, int M, int K, void* workspace, cudaStream_t st);
int tc_gemm(const TcGemmArgs& a, cudaStream_t st);

// The current device's error word of the API's tensor-core GEMMs (allocated
// and zeroed on first use; null on failure), and its check: AAEDN_ETIMEOUT
// (and the word cleared) when a bounded wait of one of them ran out.
unsigned* tc_api_err_word();
int tc_api_err_check();

} // namespace aaedn_dev
