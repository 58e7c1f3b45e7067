/*
 * oracle.h — CPU restatement of Aaedn's token loop.
 *
 * TEST INFRASTRUCTURE ONLY. This library is the checker for the CUDA path:
 * only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg may
 * load it. Nothing in the product library links, loads or calls it.
 *
 * Every function names the reference file:line it restates (paths are
 * relative to the reference project root). Where the reference is defective
 * the oracle implements the canonical choice (D1..D8) that the CUDA path also
 * implements; each such place says which decision applies:
 *   D1 scales are IEEE fp16 bit patterns on the model path
 *      (tools/convert_model.py:41,49,55); the raw dequant_4bit API keeps the
 *      integer cast of src/dequant.cpp:19.
 *   D2 weights are [out][in] row-major, 32-element quant blocks run along one
 *      row (flat order of an [out,in] tensor, tools/convert_model.py:107).
 *   D3 RoPE: rotate-half pairs (i, i+hd/2) as src/rope.cpp:50-60, angle
 *      pos * theta^(-2i/hd), fp64 -> fp32 tables, every head at the token's
 *      absolute position.
 *   D4 attention is causal MHA/GQA over the cache with the head index,
 *      scale 1/sqrt(hd) (src/transformer.cpp:198), expf.
 *   D5 KV append at the sequence length (not slot 0, src/kvcache.cpp:43).
 *   D6 SwiGLU = silu(g) * u with silu(x) = x / (1 + exp(-x)) (src/ffn.cpp:15).
 *   D7 every token of the input is processed from the current position.
 *   D8 separate final-norm gain, eps 1e-6, no biases, fp32 embedding/lm_head,
 *      greedy = argmax with ties to the lowest id.
 *
 * Parity pins: the quantizer is checked against the reference's own Python
 * function (tests/golden/), and dequant/rmsnorm/rope/attention/ffn_swiglu
 * against the reference sources compiled from source into oracle/_ref.
 */
#ifndef AAEDN_ORACLE_H
#define AAEDN_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- fp16 helpers ------------------------------------------------------ */
float or_f16_to_f32(uint16_t h);
uint16_t or_f64_to_f16(double d); /* round to nearest even, as numpy float16() */

/* ---- quantizer: tools/convert_model.py:24-55 --------------------------- */
void or_quantize_q4(const float* x, size_t n, uint8_t* data, uint16_t* scales);

/* ---- dequant ------------------------------------------------------------ */
/* src/dequant.cpp:7-28 (integer cast of the u16 scale, zero output when
 * data/scales are null or scales[0] == 0). */
void or_dequant_4bit(const uint8_t* data, const uint16_t* scales, float* out, size_t n);
/* D1 variant: scale decoded as IEEE fp16. Same null handling. */
void or_dequant_4bit_f16(const uint8_t* data, const uint16_t* scales, float* out, size_t n);

/* ---- canonical block-quant matmul (D1, D2) ------------------------------
 * out[m*ldc + n] = sum_k in[m*lda + k] * (code(n,k) * scale(n, k/32)),
 * k ascending, one fp32 accumulator per output (the loop form of
 * src/ffn.cpp:36-45). Weight row n starts at byte n*ldb/2 and scale n*ldb/32.
 * scale_kind 0 = fp16 bits (D1), 1 = integer cast (src/dequant.cpp:19). */
void or_q4_matmul(const float* in, const uint8_t* w, const uint16_t* s, float* out, size_t M, size_t N,
                  size_t K, size_t lda, size_t ldb, size_t ldc, int scale_kind);
/* fp32 matmul out[m*ldc+n] = sum_k in[m*lda+k] * w[n*ldw+k] (lm_head,
 * src/transformer.cpp:232-238). */
void or_f32_matmul(const float* in, const float* w, float* out, size_t M, size_t N, size_t K, size_t lda,
                   size_t ldw, size_t ldc);

/* ---- rmsnorm: src/rmsnorm.cpp:8-51 -------------------------------------- */
void or_rmsnorm(const float* in, float* out, const float* w, size_t n, float eps);

/* ---- RoPE ---------------------------------------------------------------- */
/* src/rope.cpp:8-34 (reference table formula freq = 10000 / 2^(i/half)). */
void or_rope_tables_ref(float* cos_t, float* sin_t, size_t max_seq, size_t head_dim);
/* D3 table: angle = pos * theta^(-2i/hd), computed in fp64, stored fp32. */
void or_rope_tables(float* cos_t, float* sin_t, size_t max_seq, size_t head_dim, double theta);
/* src/rope.cpp:36-63: rows 0..seq_len-1, row pos rotated by table row pos. */
void or_rope_apply(float* q, float* k, size_t seq_len, size_t head_dim, const float* cos_t,
                   const float* sin_t);

/* ---- attention: src/attention.cpp:10-84 with the head index (D4) ---------
 * k_cache/v_cache rows are tokens of n_heads*head_dim floats; segments is
 * (start_token, length) pairs. For n_heads == 1 this is the reference
 * function exactly. */
void or_attention(const float* q, const float* k_cache, const float* v_cache, const uint32_t* segments,
                  size_t num_segments, float* out, size_t n_heads, size_t head_dim, float scale);

/* ---- ffn with the reference's own semantics: src/ffn.cpp:18-77 -----------
 * Pin only: g*silu(g)*u, scale index j/32 (per 32 rows), integer cast. */
void or_ffn_swiglu_refsem(const float* in, float* out, size_t batch, size_t hidden, size_t ffn,
                          const uint8_t* gate, const uint8_t* up, const uint8_t* down, const uint16_t* gs,
                          const uint16_t* us, const uint16_t* ds);

/* ---- FNV-1a and the .abn v2 loader checks: src/quant.cpp:12-119 ---------- */
uint32_t or_fnv1a32(const uint8_t* p, size_t n, uint32_t h);
/* Returns 1 when the reference loader would accept the file image, else 0. */
int or_abn_v2_accepts(const uint8_t* file, size_t size);

/* ---- model oracle: src/transformer.cpp:128-243 with D1..D8 --------------- */
typedef struct {
    uint32_t dim, n_layers, n_heads, n_kv_heads, head_dim, ffn_dim, vocab, max_seq;
    double rope_theta;
    float eps;
} or_config;

typedef struct {
    const uint8_t* data;
    const uint16_t* scales; /* fp16 bits (D1) */
} or_q4;

typedef struct {
    const float* embedding;  /* [vocab][dim] */
    const float* final_norm; /* [dim] */
    const float* lm_head;    /* [vocab][dim] */
    const float* const* attn_norm; /* [L] -> [dim] */
    const float* const* ffn_norm;  /* [L] -> [dim] */
    const or_q4* wq; /* [L] -> [n_heads*hd][dim] */
    const or_q4* wk; /* [L] -> [n_kv*hd][dim] */
    const or_q4* wv; /* [L] -> [n_kv*hd][dim] */
    const or_q4* wo; /* [L] -> [dim][n_heads*hd] */
    const or_q4* wg; /* [L] -> [ffn][dim] */
    const or_q4* wu; /* [L] -> [ffn][dim] */
    const or_q4* wd; /* [L] -> [dim][ffn] */
} or_weights;

typedef struct or_model or_model;

or_model* or_model_create(const or_config* cfg, const or_weights* w);
void or_model_destroy(or_model* m);
void or_model_reset(or_model* m);
uint32_t or_model_pos(const or_model* m);
/* One token at the current position (D7); logits [vocab]; hidden_out, when
 * not null, receives the residual stream after every layer [L][dim]. */
int or_model_step(or_model* m, uint32_t token, float* logits, float* hidden_out);
/* Greedy argmax, ties to the lowest id (D8). */
uint32_t or_argmax(const float* v, size_t n);
/* Prompt then greedy decode; out_tokens receives n_new ids. Returns 0 ok. */
int or_model_generate(or_model* m, const uint32_t* prompt, size_t n_prompt, size_t n_new,
                      uint32_t* out_tokens, float* last_logits);
/* The library's seeded synthetic generator, restated (N(0, std) fp32 from
 * splitmix64 + Box-Muller keyed by (seed, tensor id, index); uniform token
 * ids in [0, vocab)). Identical outputs to aaedn_synth_normal /
 * aaedn_synth_tokens, so tests and the CPU baseline need not load the
 * library to build the same model. */
void or_synth_normal(uint64_t seed, uint64_t id, float std_dev, float* out, size_t n);
void or_synth_tokens(uint64_t seed, uint64_t id, uint32_t vocab, uint32_t* out, size_t n);
/* Timing aid: jump to position pos with synthetic K/V rows below it. */
int or_model_seek(or_model* m, uint32_t pos);
/* Threads the OpenMP loops may use (0 = library default). */
void or_set_threads(int n);
int or_get_threads(void);

#ifdef __cplusplus
}
#endif
#endif
