/*
 * aaedn_b200.h — C ABI of the B200 (sm_100a) token loop.
 *
 * Plain pointers and sizes only. Every entry point returns an int status
 * (AAEDN_OK = 0, negative on failure) and never aborts; the message of the
 * last failure on the calling thread is aaedn_last_error(). Pointers named
 * d_* are device pointers (cudaMalloc / the model's arena); h_* are host
 * pointers. `stream` is a cudaStream_t passed as void* (NULL = legacy default
 * stream). Kernels are asynchronous on that stream unless the entry point
 * says it synchronises.
 *
 * Each declaration names the reference interface it replaces
 * (file:line in the reference project). The C++ API that mirrors the
 * reference headers (namespace aaedn, project-aaedn_b200/host/include) is a
 * thin layer over these functions.
 */
#ifndef AAEDN_B200_H
#define AAEDN_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define AAEDN_OK 0
#define AAEDN_EINVAL (-1)     /* bad argument (null, size, alignment, host pointer) */
#define AAEDN_ECUDA (-2)      /* CUDA runtime error */
#define AAEDN_ETIMEOUT (-3)   /* a bounded device wait ran out */
#define AAEDN_EFORMAT (-4)    /* model/quant file rejected */
#define AAEDN_ENOMEM (-5)     /* allocation or arena overflow */
#define AAEDN_EUNSUPPORTED (-6)
#define AAEDN_ESTATE (-7)     /* object not initialised / sequence full */

/* scale_kind for the block-quant entry points */
#define AAEDN_SCALE_F16 0     /* u16 holds IEEE fp16 bits (tools/convert_model.py:49) */
#define AAEDN_SCALE_U16INT 1  /* u16 cast to float as an integer (src/dequant.cpp:19) */

const char* aaedn_last_error(void);
int aaedn_version(void);
/* Number of kernels this library has launched in this process (all entry
 * points, graph replays counted per kernel node). */
uint64_t aaedn_kernel_launches(void);

/* ---- device memory helpers (plain cudaMalloc / cudaMemcpy) -------------- */
int aaedn_dev_alloc(void** d_ptr, size_t bytes);
int aaedn_dev_free(void* d_ptr);
int aaedn_memcpy_h2d(void* d_dst, const void* h_src, size_t bytes, void* stream);
int aaedn_memcpy_d2h(void* h_dst, const void* d_src, size_t bytes, void* stream);
int aaedn_memcpy_d2d(void* d_dst, const void* d_src, size_t bytes, void* stream);
int aaedn_stream_sync(void* stream);
int aaedn_device_sync(void);

/* ---- host-side quant tools (no GPU needed) ------------------------------- */
/* tools/convert_model.py:36-55 quantize_block_4bit_unsigned, bit-exact:
 * 32-element blocks in flat order, scale = fp16(max|x|/7), codes
 * clip(rint(x/scale), 0, 15), low nibble = even element. data: (n+1)/2 B,
 * scales: ceil(n/32) u16. Multi-threaded. */
int aaedn_quantize_q4(const float* h_x, size_t n, uint8_t* h_data, uint16_t* h_scales);
/* tools/convert_model.py:16-21 / src/quant.cpp:12-20 FNV-1a 32. */
uint32_t aaedn_fnv1a32(const uint8_t* h_p, size_t n, uint32_t seed);
/* Seeded synthetic tensors: N(0, std) fp32 from a counter-based generator
 * keyed by (seed, tensor_id, index); identical on every host. */
int aaedn_synth_normal(uint64_t seed, uint64_t tensor_id, float std_dev, float* h_out, size_t n);
/* Uniform token ids in [0, vocab). */
int aaedn_synth_tokens(uint64_t seed, uint64_t stream_id, uint32_t vocab, uint32_t* h_out, size_t n);
/* RoPE tables [max_seq][hd/2]. formula 0: src/rope.cpp:26 (freq =
 * 10000/2^(i/half), fp32 as the reference); formula 1: pos*theta^(-2i/hd)
 * in fp64 rounded to fp32 (the model path). */
int aaedn_rope_table(float* h_cos, float* h_sin, size_t max_seq, size_t head_dim, double theta, int formula);

/* ---- tokenizer (.abt v2; host only, no GPU needed) ----------------------- */
/* src/tokenizer.cpp:32-158 tokenizer_load: reads an .abt v2 file (64-byte
 * header "<8sIQI4I24s", magic "AAEDNTOK", FNV-1a 32 of the payload; the
 * payload's string block, u32 offsets and u16 merge-rule pairs) with the
 * reference's accept/reject decisions (AAEDN_EFORMAT when rejected). The
 * handle owns host copies of the tables and a pair -> rule lookup table. */
typedef struct aaedn_tokenizer aaedn_tokenizer;
int aaedn_tokenizer_load(const char* path, aaedn_tokenizer** out);
/* The same from a file image already in host memory. */
int aaedn_tokenizer_from_bytes(const uint8_t* h_file, size_t n, aaedn_tokenizer** out);
void aaedn_tokenizer_free(aaedn_tokenizer* t);
/* h_info[5] = vocab_size, merge_count, max_token_bytes, format_version,
 * payload_checksum (include/tokenizer.hpp:19-30). */
int aaedn_tokenizer_info(const aaedn_tokenizer* t, uint32_t* h_info);
/* src/tokenizer.cpp:169-239 tokenizer_encode: one id per byte of the
 * NUL-terminated text, merged by the rules in the reference's order (merged
 * pair = vocab_size + rule number), 32765 (BOS) first when add_bos. At most
 * strlen(text) + add_bos ids. h_ids == NULL (cap 0): only *n_ids is set. */
int aaedn_tokenizer_encode(const aaedn_tokenizer* t, const char* text, int add_bos, uint32_t* h_ids, size_t cap,
                           size_t* n_ids);
/* src/tokenizer.cpp:241-257 tokenizer_decode: the strings of the ids,
 * concatenated (32766, 32767 and ids >= vocab_size add nothing); *n_bytes =
 * its length, and h_text (cap > length) gets it with a NUL after it.
 * h_text == NULL (cap 0): only *n_bytes is set. */
int aaedn_tokenizer_decode(const aaedn_tokenizer* t, const uint32_t* h_ids, size_t n, char* h_text, size_t cap,
                           size_t* n_bytes);

/* ---- .abn model files (tools/convert_model.py:138, src/quant.cpp:31-119) -- */
/* The 64-byte little-endian header "<8sIQI6IB15s": magic "AAEDNMDL",
 * version, payload_size, payload_checksum (FNV-1a 32 of the payload),
 * n_layers, n_heads, head_dim, vocab_size, hidden_dim, ffn_dim, quant_type. */
typedef struct {
    uint32_t version;
    uint64_t payload_size;
    uint32_t payload_checksum;
    uint32_t n_layers, n_heads, head_dim, vocab_size, hidden_dim, ffn_dim;
    uint8_t quant_type;
} aaedn_abn_header;
/* Reads and checks the header as quant_load does (src/quant.cpp:50-72):
 * magic, version 2 and payload_size == hidden^2/2 + hidden^2/16.
 * AAEDN_EFORMAT when the file is short or rejected. */
int aaedn_abn_read_header(const char* path, aaedn_abn_header* h_out);
/* Reads the payload after a header accepted by aaedn_abn_read_header into
 * h_data (hidden^2/2 bytes) and h_scales (hidden^2/32 u16) and checks the
 * FNV-1a checksum (src/quant.cpp:87-111). AAEDN_EFORMAT on a short file or a
 * checksum mismatch. */
int aaedn_abn_read_payload(const char* path, const aaedn_abn_header* h_hdr, uint8_t* h_data, uint16_t* h_scales);


/* ---- kernels (device pointers) ------------------------------------------ */
/* include/dequant.hpp:10 dequant_4bit (src/dequant.cpp:7-28): out[i] =
 * code(i) * scale(i/32); all-zero output when data/scales are null or
 * scales[0] == 0 (checked on the device). Bit-exact. */
int aaedn_cu_dequant_4bit(const uint8_t* d_data, const uint16_t* d_scales, float* d_out, size_t n,
                          int scale_kind, void* stream);

/* include/fused_matmul.hpp:13 fused_matmul: out[m*ldc+n] = sum_k
 * in[m*lda+k] * code(n,k) * scale(n,k/32). Weights are [N][K] rows of ldb
 * codes (ldb/2 bytes, ldb/32 scales per row), K and ldb multiples of 32.
 * M == 0 or N == 0 or K == 0 is a no-op (src/fused_matmul.cpp:76-77). */
int aaedn_cu_fused_matmul(const float* d_in, const uint8_t* d_w, const uint16_t* d_scales, float* d_out,
                          size_t M, size_t N, size_t K, size_t lda, size_t ldb, size_t ldc, int scale_kind,
                          void* stream);

/* fused_matmul on weights repacked into the tile-major layout the model
 * streams (the same 32-code blocks and fp16 scales, reordered so that each
 * 16-row group's K range is one run of 1152-byte tiles): M == 1 runs the
 * decode GEMV engine, M > 1 the tcgen05 GEMM. N % 16 == 0, K % 128 == 0,
 * K <= 32768; d_in is [M][K], d_out [M][N] (dense). The repack is host
 * side: h_out holds aaedn_q4_tiled_bytes(N, K) bytes (codes + fp16 scales
 * of aaedn_quantize_q4's row-major output). */
size_t aaedn_q4_tiled_bytes(size_t N, size_t K);
int aaedn_q4_repack_tiled(const uint8_t* h_codes, const uint16_t* h_scales, size_t N, size_t K, uint8_t* h_out);
int aaedn_cu_fused_matmul_tiled(const float* d_in, const uint8_t* d_tiled, float* d_out, size_t M, size_t N,
                                size_t K, void* stream);

/* fp32 weights: out[m*ldc+n] = sum_k in[m*lda+k]*w[n*ldw+k] (the lm_head
 * product of src/transformer.cpp:232-238). */
int aaedn_cu_f32_matmul(const float* d_in, const float* d_w, float* d_out, size_t M, size_t N, size_t K,
                        size_t lda, size_t ldw, size_t ldc, void* stream);

/* include/rmsnorm.hpp:10 rmsnorm (src/rmsnorm.cpp:8-51). */
int aaedn_cu_rmsnorm(const float* d_in, float* d_out, const float* d_w, size_t n, float eps, void* stream);

/* include/rope.hpp:21 rope_apply (src/rope.cpp:36-63): rows 0..seq_len-1 of
 * q and k ([seq_len][head_dim]) rotated by table rows 0..seq_len-1. */
int aaedn_cu_rope_apply(float* d_q, float* d_k, size_t seq_len, size_t head_dim, const float* d_cos,
                        const float* d_sin, void* stream);

/* include/attention.hpp:13 attention (src/attention.cpp:10-84, head index
 * added): k/v rows are tokens of n_heads*head_dim floats; h_segments holds
 * num_segments (start_token, length) pairs on the HOST (at most 64, the
 * reference keeps 32 per agent: src/kvcache.cpp:33). */
int aaedn_cu_attention(const float* d_q, const float* d_k, const float* d_v, const uint32_t* h_segments,
                       size_t num_segments, float* d_out, size_t n_heads, size_t head_dim, float scale,
                       void* stream);

/* include/ffn.hpp:12 ffn_swiglu (src/ffn.cpp:18-77): out[b] = W_down *
 * act(W_gate * in[b], W_up * in[b]) for batch rows of hidden floats; weights
 * [out][in] row-major 4-bit codes (gate/up: ffn x hidden, down: hidden x
 * ffn). AAEDN_FFN_MODEL: fp16 scale per (row, 32 inputs), act = silu(g)*u
 * (the model path). AAEDN_FFN_REFERENCE: what src/ffn.cpp:41-72 computes
 * (scale of output row j = scales[j/32] as an integer, act = g*silu(g)*u).
 * Null weights or scales give zero output (src/ffn.cpp:22-27). */
#define AAEDN_FFN_MODEL 0
#define AAEDN_FFN_REFERENCE 1
int aaedn_cu_ffn_swiglu(const float* d_in, float* d_out, size_t batch, size_t hidden, size_t ffn,
                        const uint8_t* d_gate, const uint8_t* d_up, const uint8_t* d_down,
                        const uint16_t* d_gate_scales, const uint16_t* d_up_scales, const uint16_t* d_down_scales,
                        int semantics, void* stream);

/* Next-token sampling (docs/mpd.md:539-554; src/main.cpp:214-247 is the
 * reference's softmax-and-draw without temperature or top-p, walking ids in
 * index order where this walks them in the spec's sorted order):
 * temperature T, nucleus top_p, multinomial draw with the caller's uniform
 * variate u in [0, 1) (the reference's rand() / RAND_MAX). T <= 0 is greedy
 * (argmax, ties to the lowest id). Otherwise p_i = exp((l_i - max) / T); the
 * tokens sorted by p descending (ties: lower id first) are kept up to and
 * including the first whose cumulative sum reaches top_p * sum(p); the token
 * returned is the first kept one whose cumulative sum reaches u times the
 * kept mass. Masses are summed in fp64. Writes one uint32 to d_token. */
int aaedn_cu_sample(const float* d_logits, uint32_t vocab, float temperature, float top_p, float u,
                    uint32_t* d_token, void* stream);

/* No counterpart in the reference. The same attention as
 * aaedn_cu_attention for callers that cannot let a library allocate device
 * memory (for example an application that hands all device memory to one
 * fixed pool at startup and forbids allocation afterwards, the rule the
 * reference states in docs/sdd.md:78 and README.md:18). It calls no
 * cudaMalloc or cudaFree: its scratch (the per-split partial results and the
 * split counters) is a fixed AAEDN_ATTN_NOALLOC_SCRATCH_BYTES array that
 * every GPU loading this library holds until the process exits. Shapes whose
 * scratch would not fit (n_heads > 1024, or n_heads*(head_dim+2)*4 bytes
 * above the partial area) are rejected with AAEDN_EINVAL. The first call on
 * each device looks up the array's device address: make that first call
 * before any stream capture. All calls share the one array: calls that
 * overlap on the GPU (another stream, another thread) race; serialise them. */
#define AAEDN_ATTN_NOALLOC_SCRATCH_BYTES (1u << 20)
int aaedn_cu_attention_noalloc(const float* d_q, const float* d_k, const float* d_v, const uint32_t* h_segments,
                               size_t num_segments, float* d_out, size_t n_heads, size_t head_dim, float scale,
                               void* stream);

/* ---- the token loop ------------------------------------------------------
 * include/transformer.hpp:15-44 Transformer / transformer_init /
 * transformer_forward. One model owns one device arena (a single
 * cudaMalloc at creation: the reference's no-allocation-after-startup rule,
 * docs/mpd.md:59), the weights, a paged fp32 KV cache and one stream. */
typedef struct aaedn_model aaedn_model;

typedef struct {
    uint32_t dim, n_layers, n_heads, n_kv_heads, head_dim, ffn_dim, vocab, max_seq;
    float rope_theta;
    float eps;
} aaedn_model_config;

/* Host weights of one layer in logical order, [out][in] rows, quantized
 * with aaedn_quantize_q4 (fp16 scales). */
typedef struct {
    const uint8_t *wq, *wk, *wv, *wo, *wg, *wu, *wd;
    const uint16_t *sq, *sk, *sv, *so, *sg, *su, *sd;
    const float *attn_norm, *ffn_norm; /* [dim] */
} aaedn_layer_host;

int aaedn_model_create(const aaedn_model_config* cfg, aaedn_model** out);

/* ---- tensor parallelism over the GPUs of one node -------------------------
 * No counterpart in the reference (its token loop is single-process CPU);
 * this is the multi-GPU decomposition of src/transformer.cpp:128-243. Rank r
 * of tp_size (1, 2, 4, 8; one process per GPU, that GPU current) holds heads
 * [r*H/T, (r+1)*H/T) and their KV cache, gate/up rows [r*F/T, ...), the
 * matching input columns of o and down, and lm_head rows [r*ceil(V/T), ...).
 * set_layer / set_globals / synthesize take the WHOLE tensors on every rank;
 * config_get returns the whole model's dims. After o and down the ranks'
 * partial sums are added through each other's memory (CUDA IPC over NVLink):
 * every rank exports its handle with aaedn_model_tp_handle, gathers all
 * tp_size handles in rank order (any host channel) and passes them to
 * aaedn_model_tp_connect before its first step. All ranks then run the same
 * calls with the same tokens (lockstep); forward's h_logits receives this
 * rank's vocabulary slice. Waits between ranks are bounded (2 s; a timeout
 * reports AAEDN_ETIMEOUT-class failure through the step's error). Destroy on
 * every rank only after all ranks are done stepping. */
#define AAEDN_TP_HANDLE_BYTES 64
/* The share of rank tp_rank (host only, no GPU): heads [q_head0, +n_heads),
 * kv heads [kv_head0, +n_kv_heads), ffn rows [ffn_row0, +ffn_dim), lm_head
 * rows / token ids [vocab0, +vocab); o and down take input columns
 * [q_head0*head_dim, +n_heads*head_dim) and [ffn_row0, +ffn_dim), padded to
 * o_k / down_k columns on the device. AAEDN_EINVAL if the shape does not
 * divide (n_kv_heads % T, ffn_dim % (32 T)). */
typedef struct {
    uint32_t n_heads, n_kv_heads, ffn_dim, vocab;
    uint32_t q_head0, kv_head0, ffn_row0, vocab0;
    uint32_t o_k, down_k;
} aaedn_tp_plan;
int aaedn_tp_plan_get(const aaedn_model_config* cfg, uint32_t tp_rank, uint32_t tp_size, aaedn_tp_plan* out);
int aaedn_model_create_tp(const aaedn_model_config* cfg, uint32_t tp_rank, uint32_t tp_size, aaedn_model** out);
int aaedn_model_tp_handle(aaedn_model* m, uint8_t* h_handle);
int aaedn_model_tp_connect(aaedn_model* m, const uint8_t* h_handles);
int aaedn_model_destroy(aaedn_model* m);
int aaedn_model_config_get(const aaedn_model* m, aaedn_model_config* out);
void* aaedn_model_stream(aaedn_model* m);
/* Device bytes the arena holds. */
size_t aaedn_model_arena_bytes(const aaedn_model* m);
int aaedn_model_set_layer(aaedn_model* m, uint32_t layer, const aaedn_layer_host* w);
/* embedding [vocab][dim], final_norm [dim], lm_head [vocab][dim], fp32 host. */
int aaedn_model_set_globals(aaedn_model* m, const float* h_embedding, const float* h_final_norm,
                            const float* h_lm_head);
/* Whole-model files: the per-layer layout of docs/mpd.md:497-499 (RMSNorm
 * scale fp32 [dim] | QKV weight | QKV bias fp32 | O weight | FFN gate | FFN
 * up | FFN down | RMSNorm 2 scale fp32 [dim]; a weight = row-major 4-bit
 * codes then its u16 fp16-bit scales; QKV rows are the q heads, then k, then
 * v), followed by the final-norm gain fp32 [dim], the embedding and the
 * lm_head fp32 [vocab][dim]. The reference's converter does not write it yet
 * (tools/convert_model.py:121-126 writes one matrix), so the header marks it
 * version 3 and keeps what the documented header lacks in its reserved
 * bytes: n_kv_heads (u32, offset 49), rope_theta (f32, 53), eps (f32, 57).
 * Reads and checks the header and returns the model shape (max_seq 0: the
 * caller chooses the context). AAEDN_EFORMAT when the file is rejected. */
int aaedn_abn_model_read_header(const char* path, aaedn_abn_header* h_out, aaedn_model_config* cfg_out);
/* Every weight of a whole-model file (aaedn_abn_model_read_header) into a
 * model of the same shape (a tensor-parallel rank keeps its share): the
 * FNV-1a checksum of the payload is checked first, then the layers are read
 * one at a time. A nonzero QKV bias is AAEDN_EUNSUPPORTED (the model has
 * none, src/transformer.cpp:112-117). No counterpart in the reference (its
 * transformer_init fills weights with constants and rand()). */
int aaedn_model_load_abn(aaedn_model* m, const char* path);
/* Writes a whole-model file in the layout aaedn_model_load_abn reads, from
 * host tensors: layers[n_layers] (quantized with aaedn_quantize_q4, fp16
 * scales; null norm gains are written as 1.0), the fp32 embedding and lm_head
 * [vocab][dim] and the final-norm gain [dim] (null: 1.0); the QKV bias is
 * written as zeros. The converter role of tools/convert_model.py:121-150
 * (which writes one matrix in the version-2 header) for the whole model. */
int aaedn_abn_model_write(const char* path, const aaedn_model_config* cfg, const aaedn_layer_host* layers,
                          const float* h_embedding, const float* h_final_norm, const float* h_lm_head);
/* Fill every weight from the seeded generator (N(0,0.02) linear weights
 * quantized with the block quantizer; fp32 embedding and lm_head; norm gains
 * 1.0). Tensor ids: embedding 0, lm_head 1, layer l: 16 + 8l + {q,k,v,o,g,u,d}.
 * Multi-threaded on the host, then uploaded. */
int aaedn_model_synthesize(aaedn_model* m, uint64_t seed);
/* Start a new sequence at position 0 (the KV cache content is discarded). */
int aaedn_model_reset(aaedn_model* m);
uint32_t aaedn_model_pos(aaedn_model* m);
/* src/transformer.cpp:128-243 transformer_forward: process the n tokens at
 * the current position (D7), return the last token's logits to h_logits
 * [vocab] (may be NULL). Synchronises. */
int aaedn_model_forward(aaedn_model* m, const uint32_t* h_tokens, size_t n, float* h_logits);
/* Prompt, then greedy decode of n_new tokens entirely on the device (argmax
 * ties to the lowest id). Synchronises and copies the ids to h_out. */
int aaedn_model_generate(aaedn_model* m, const uint32_t* h_prompt, size_t n_prompt, size_t n_new,
                         uint32_t* h_out);
/* Device-resident greedy steps with no host synchronisation (one CUDA graph
 * replay per step); the sequence must already hold at least one token. */
int aaedn_model_decode_steps(aaedn_model* m, size_t n_steps);
/* Move the sequence back to position pos (1 <= pos <= current): the cache
 * below pos stays valid and decoding resumes from the greedy token of the
 * last step (the reference REPL's /reset, src/main.cpp:83-86, keeps nothing;
 * this keeps the prefix). */
int aaedn_model_rewind(aaedn_model* m, uint32_t pos);
/* Tracing: one decode step replayed as a CUDA graph with an event between
 * every kernel; h_ms[i] receives the device time of kernel i in launch order
 * (per layer: qkv, attention, o, gate/up, down; then lm_head). cap is the
 * capacity of h_ms; returns the kernel count through *n_out. */
int aaedn_model_profile_step(aaedn_model* m, float* h_ms, uint32_t cap, uint32_t* n_out);
/* Tracing: device time of sub-graphs of one decode step replayed `reps`
 * times back to back with the decode graph's launch setup; h_ms (>= 8
 * entries) receives ms per step of: all kernels, the dequant-GEMVs, qkv,
 * attention, o, gate/up, down, lm_head. Leaves the KV cache and hidden state
 * undefined (rewind or reset afterwards). */
int aaedn_model_profile_parts(aaedn_model* m, uint32_t reps, float* h_ms, uint32_t cap);
/* Tracing of the per-kernel decode step: one step replayed with globaltimer
 * stamps (ns) per CTA; h_stamps [5 * n_layers + 1][1024][4]: per launch (qkv,
 * attention, o, gate/up, down of each layer, then lm_head) and CTA slot c <
 * 160: entry, operand ready, [GEMV: previous kernel complete; attention: its
 * token loop done], exit (0 where a kernel records no such event); GEMV
 * launches also hold, from slot 160 on, consumer warp 0's (arrived, released)
 * stamps of chunks 0..23 of CTAs 0..7 (48 words per CTA); h_grid [5 *
 * n_layers + 1]: CTAs per launch (0: not traced). Single-GPU models only; the
 * position is left where it was. No counterpart in the reference. */
int aaedn_model_trace_kernels(aaedn_model* m, uint64_t* h_stamps, size_t cap, uint32_t* h_grid, size_t cap_grid);
/* Synchronises and reports the sticky device-side error of the decode state
 * (AAEDN_ESTATE: a position past the cache; AAEDN_ETIMEOUT: a bounded device
 * wait ran out). forward and generate check it themselves; decode_steps does
 * not synchronise, so call this after it. */
int aaedn_model_status(aaedn_model* m);
/* The greedy token of the last step (the next input), from the device
 * state (synchronises). */
int aaedn_model_next_token(aaedn_model* m, uint32_t* h_token);
/* Kernels launched by one decode step. */
uint32_t aaedn_model_kernels_per_step(const aaedn_model* m);
/* Prompt tokens one prefill chunk takes through the tensor-core GEMMs
 * (forward / generate with more than one token); 0 when the model runs its
 * prompt as one decode step per token (tensor-parallel ranks, and matrix
 * shapes without the tile-major layout: K % 128 or N % 16 nonzero). No
 * counterpart in the reference (src/transformer.cpp:146 processes one token). */
uint32_t aaedn_model_prefill_rows(const aaedn_model* m);
/* Copy the last step's logits ([vocab]) / the greedy tokens generated so far. */
int aaedn_model_logits(aaedn_model* m, float* h_logits);
int aaedn_model_tokens(aaedn_model* m, uint32_t* h_out, size_t n);
/* Debug path (eager launches): one token, the residual stream after every
 * layer to h_hidden [n_layers][dim] and the logits to h_logits. */
int aaedn_model_forward_debug(aaedn_model* m, uint32_t token, float* h_hidden, float* h_logits);

/* ---- batched sequences over a shared, paged KV cache -----------------------
 * The per-agent view of the reference's cache (src/kvcache.cpp:15-60:
 * segment_tables per agent) and its branch protocol (docs/sdd.md:206-215:
 * a child branch continues from its parent's tokens, a pruned branch's
 * storage is released; src/agent.cpp:107-140 agent_diverge / agent_merge)
 * on the device. A batched model holds up to max_seqs sequences whose K/V
 * rows live in one pool of pages of 64 tokens (kv_tokens tokens in all); a
 * sequence is a page table. aaedn_seq_fork gives the child the parent's
 * pages (shared, counted, nothing copied); the first append of either into a
 * page they share copies that page first (copy on write); aaedn_seq_close
 * releases the pages no other sequence holds. aaedn_model_step_batch runs
 * one token of each listed sequence through one pass: every matrix product
 * is the tensor-core GEMM over the batch's rows, attention reads each row's
 * own pages. Weights go in with aaedn_model_set_layer / set_globals /
 * synthesize / load_abn as for aaedn_model_create; the single-sequence calls
 * (forward, generate, decode_steps) are not available on a batched model. No
 * counterpart in the reference beyond the cited bookkeeping (its
 * transformer_forward runs one token of one sequence). */
int aaedn_model_create_batched(const aaedn_model_config* cfg, uint32_t max_seqs, uint64_t kv_tokens,
                               aaedn_model** out);
/* A new empty sequence (AAEDN_ENOMEM when max_seqs are open). */
int aaedn_seq_open(aaedn_model* m, uint32_t* seq);
/* A new sequence that continues from parent's tokens, sharing its pages. */
int aaedn_seq_fork(aaedn_model* m, uint32_t parent, uint32_t* child);
/* Closes the sequence (prune): its pages go back to the pool unless another
 * sequence still holds them. */
int aaedn_seq_close(aaedn_model* m, uint32_t seq);
int aaedn_seq_len(aaedn_model* m, uint32_t seq, uint32_t* len);
/* Pages in the pool and how many are free. */
int aaedn_model_kv_pages(aaedn_model* m, uint32_t* total, uint32_t* free_pages);
/* n tokens appended to one sequence through the prefill path; h_logits
 * [vocab] (may be NULL) and h_next (may be NULL) receive the last token's
 * logits and greedy next token. Synchronises. */
int aaedn_seq_prefill(aaedn_model* m, uint32_t seq, const uint32_t* h_tokens, size_t n, float* h_logits,
                      uint32_t* h_next);
/* One token for each of n distinct open sequences h_seqs[i] (h_tokens[i] at
 * the sequence's next position), all in one batched pass; h_logits
 * [n][vocab] and h_next [n] (either may be NULL) receive each row's logits
 * and greedy token. Synchronises. */
int aaedn_model_step_batch(aaedn_model* m, const uint32_t* h_seqs, const uint32_t* h_tokens, size_t n,
                           float* h_logits, uint32_t* h_next);

#ifdef __cplusplus
}
#endif
#endif
