"""ctypes binding of libaaedn_b200.so (the C ABI in include/aaedn_b200.h).

The CUDA library is the only compute path: there is no CPU fallback. If the
shared library is missing this module raises on import of any compute
entry point; build it with ``python project-aaedn_b200/build.py``.

Device buffers can be any CUDA allocation (torch tensors are convenient:
pass ``t.data_ptr()``); host buffers are numpy arrays.
"""
import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
# AAEDN_B200_LIB: another build of the library (same C ABI) to load instead
LIB_PATH = os.environ.get("AAEDN_B200_LIB") or os.path.join(HERE, "libaaedn_b200.so")

OK = 0
EINVAL, ECUDA, ETIMEOUT, EFORMAT, ENOMEM, EUNSUPPORTED, ESTATE = -1, -2, -3, -4, -5, -6, -7
SCALE_F16, SCALE_U16INT = 0, 1

_vp = ctypes.c_void_p
_sz = ctypes.c_size_t
_u32 = ctypes.c_uint32
_u64 = ctypes.c_uint64
_int = ctypes.c_int
_f32 = ctypes.c_float


class AaednError(RuntimeError):
    def __init__(self, rc, msg):
        super().__init__(f"aaedn error {rc}: {msg}")
        self.rc = rc


class ModelConfig(ctypes.Structure):
    _fields_ = [("dim", _u32), ("n_layers", _u32), ("n_heads", _u32), ("n_kv_heads", _u32), ("head_dim", _u32),
                ("ffn_dim", _u32), ("vocab", _u32), ("max_seq", _u32), ("rope_theta", _f32), ("eps", _f32)]

    def as_dict(self):
        d = {k: getattr(self, k) for k, _ in self._fields_}
        return d


class AbnHeader(ctypes.Structure):
    _fields_ = [("version", _u32), ("payload_size", _u64), ("payload_checksum", _u32), ("n_layers", _u32),
                ("n_heads", _u32), ("head_dim", _u32), ("vocab_size", _u32), ("hidden_dim", _u32),
                ("ffn_dim", _u32), ("quant_type", ctypes.c_uint8)]


class TpPlan(ctypes.Structure):
    _fields_ = [(n, _u32) for n in ("n_heads", "n_kv_heads", "ffn_dim", "vocab", "q_head0", "kv_head0",
                                    "ffn_row0", "vocab0", "o_k", "down_k")]


def tp_plan(cfg, rank, size):
    """The share of tensor-parallel rank `rank` of `size` (host only)."""
    c = ModelConfig(**{k: cfg[k] for k, _ in ModelConfig._fields_})
    p = TpPlan()
    check(lib().aaedn_tp_plan_get(ctypes.byref(c), rank, size, ctypes.byref(p)))
    return {k: getattr(p, k) for k, _ in TpPlan._fields_}


class LayerHost(ctypes.Structure):
    _fields_ = [(n, _vp) for n in ("wq", "wk", "wv", "wo", "wg", "wu", "wd",
                                   "sq", "sk", "sv", "so", "sg", "su", "sd", "attn_norm", "ffn_norm")]


_lib = None


def lib():
    """The loaded shared library (raises if it was not built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"{LIB_PATH} is missing: build it with python project-aaedn_b200/build.py")
    L = ctypes.CDLL(LIB_PATH)
    sig = {
        "aaedn_last_error": ([], ctypes.c_char_p),
        "aaedn_version": ([], _int),
        "aaedn_kernel_launches": ([], _u64),
        "aaedn_dev_alloc": ([ctypes.POINTER(_vp), _sz], _int),
        "aaedn_dev_free": ([_vp], _int),
        "aaedn_memcpy_h2d": ([_vp, _vp, _sz, _vp], _int),
        "aaedn_memcpy_d2h": ([_vp, _vp, _sz, _vp], _int),
        "aaedn_stream_sync": ([_vp], _int),
        "aaedn_device_sync": ([], _int),
        "aaedn_quantize_q4": ([_vp, _sz, _vp, _vp], _int),
        "aaedn_fnv1a32": ([_vp, _sz, _u32], _u32),
        "aaedn_synth_normal": ([_u64, _u64, _f32, _vp, _sz], _int),
        "aaedn_synth_tokens": ([_u64, _u64, _u32, _vp, _sz], _int),
        "aaedn_rope_table": ([_vp, _vp, _sz, _sz, ctypes.c_double, _int], _int),
        "aaedn_cu_dequant_4bit": ([_vp, _vp, _vp, _sz, _int, _vp], _int),
        "aaedn_cu_fused_matmul": ([_vp, _vp, _vp, _vp, _sz, _sz, _sz, _sz, _sz, _sz, _int, _vp], _int),
        "aaedn_cu_f32_matmul": ([_vp, _vp, _vp, _sz, _sz, _sz, _sz, _sz, _sz, _vp], _int),
        "aaedn_tokenizer_load": ([ctypes.c_char_p, ctypes.POINTER(_vp)], _int),
        "aaedn_tokenizer_from_bytes": ([_vp, _sz, ctypes.POINTER(_vp)], _int),
        "aaedn_tokenizer_free": ([_vp], None),
        "aaedn_tokenizer_info": ([_vp, _vp], _int),
        "aaedn_tokenizer_encode": ([_vp, ctypes.c_char_p, _int, _vp, _sz, ctypes.POINTER(_sz)], _int),
        "aaedn_tokenizer_decode": ([_vp, _vp, _sz, _vp, _sz, ctypes.POINTER(_sz)], _int),
        "aaedn_q4_tiled_bytes": ([_sz, _sz], _sz),
        "aaedn_q4_repack_tiled": ([_vp, _vp, _sz, _sz, _vp], _int),
        "aaedn_cu_fused_matmul_tiled": ([_vp, _vp, _vp, _sz, _sz, _sz, _vp], _int),
        "aaedn_cu_rmsnorm": ([_vp, _vp, _vp, _sz, _f32, _vp], _int),
        "aaedn_cu_rope_apply": ([_vp, _vp, _sz, _sz, _vp, _vp, _vp], _int),
        "aaedn_cu_attention": ([_vp, _vp, _vp, _vp, _sz, _vp, _sz, _sz, _f32, _vp], _int),
        "aaedn_cu_attention_noalloc": ([_vp, _vp, _vp, _vp, _sz, _vp, _sz, _sz, _f32, _vp], _int),
        "aaedn_cu_ffn_swiglu": ([_vp, _vp, _sz, _sz, _sz, _vp, _vp, _vp, _vp, _vp, _vp, _int, _vp], _int),
        "aaedn_memcpy_d2d": ([_vp, _vp, _sz, _vp], _int),
        "aaedn_cu_sample": ([_vp, _u32, ctypes.c_float, ctypes.c_float, ctypes.c_float, _vp, _vp], _int),
        "aaedn_abn_read_header": ([ctypes.c_char_p, ctypes.POINTER(AbnHeader)], _int),
        "aaedn_abn_read_payload": ([ctypes.c_char_p, ctypes.POINTER(AbnHeader), _vp, _vp], _int),
        "aaedn_model_create": ([ctypes.POINTER(ModelConfig), ctypes.POINTER(_vp)], _int),
        "aaedn_model_create_tp": ([ctypes.POINTER(ModelConfig), _u32, _u32, ctypes.POINTER(_vp)], _int),
        "aaedn_model_tp_handle": ([_vp, _vp], _int),
        "aaedn_model_tp_connect": ([_vp, _vp], _int),
        "aaedn_model_status": ([_vp], _int),
        "aaedn_model_next_token": ([_vp, ctypes.POINTER(_u32)], _int),
        "aaedn_tp_plan_get": ([ctypes.POINTER(ModelConfig), _u32, _u32, ctypes.POINTER(TpPlan)], _int),
        "aaedn_model_destroy": ([_vp], _int),
        "aaedn_model_config_get": ([_vp, ctypes.POINTER(ModelConfig)], _int),
        "aaedn_model_stream": ([_vp], _vp),
        "aaedn_model_arena_bytes": ([_vp], _sz),
        "aaedn_model_set_layer": ([_vp, _u32, ctypes.POINTER(LayerHost)], _int),
        "aaedn_model_set_globals": ([_vp, _vp, _vp, _vp], _int),
        "aaedn_abn_model_read_header": ([ctypes.c_char_p, ctypes.POINTER(AbnHeader), ctypes.POINTER(ModelConfig)],
                                        _int),
        "aaedn_model_load_abn": ([_vp, ctypes.c_char_p], _int),
        "aaedn_abn_model_write": ([ctypes.c_char_p, ctypes.POINTER(ModelConfig), ctypes.POINTER(LayerHost), _vp, _vp,
                                   _vp], _int),
        "aaedn_model_synthesize": ([_vp, _u64], _int),
        "aaedn_model_reset": ([_vp], _int),
        "aaedn_model_pos": ([_vp], _u32),
        "aaedn_model_forward": ([_vp, _vp, _sz, _vp], _int),
        "aaedn_model_generate": ([_vp, _vp, _sz, _sz, _vp], _int),
        "aaedn_model_decode_steps": ([_vp, _sz], _int),
        "aaedn_model_kernels_per_step": ([_vp], _u32),
        "aaedn_model_prefill_rows": ([_vp], _u32),
        "aaedn_model_create_batched": ([ctypes.POINTER(ModelConfig), _u32, _u64, ctypes.POINTER(_vp)], _int),
        "aaedn_seq_open": ([_vp, ctypes.POINTER(_u32)], _int),
        "aaedn_seq_fork": ([_vp, _u32, ctypes.POINTER(_u32)], _int),
        "aaedn_seq_close": ([_vp, _u32], _int),
        "aaedn_seq_len": ([_vp, _u32, ctypes.POINTER(_u32)], _int),
        "aaedn_model_kv_pages": ([_vp, ctypes.POINTER(_u32), ctypes.POINTER(_u32)], _int),
        "aaedn_seq_prefill": ([_vp, _u32, _vp, _sz, _vp, _vp], _int),
        "aaedn_model_step_batch": ([_vp, _vp, _vp, _sz, _vp, _vp], _int),
        "aaedn_model_logits": ([_vp, _vp], _int),
        "aaedn_model_tokens": ([_vp, _vp, _sz], _int),
        "aaedn_model_forward_debug": ([_vp, _u32, _vp, _vp], _int),
        "aaedn_model_rewind": ([_vp, _u32], _int),
        "aaedn_model_profile_parts": ([_vp, _u32, _vp, _u32], _int),
        "aaedn_model_profile_step": ([_vp, _vp, _u32, ctypes.POINTER(_u32)], _int),
        "aaedn_model_trace_kernels": ([_vp, _vp, _sz, _vp, _sz], _int),
    }
    for name, (args, res) in sig.items():
        f = getattr(L, name)
        f.argtypes = args
        f.restype = res
    _lib = L
    return L


def exported_symbols():
    """Names declared in include/aaedn_b200.h that the library must export."""
    import re
    hdr = os.path.join(os.path.dirname(os.path.dirname(HERE)), "include", "aaedn_b200.h")
    txt = open(hdr).read()
    return sorted(set(re.findall(r"\b(aaedn_[a-z0-9_]+)\s*\(", txt)))


def last_error():
    return lib().aaedn_last_error().decode(errors="replace")


def check(rc):
    if rc != OK:
        raise AaednError(rc, last_error())
    return rc


def kernel_launches():
    return int(lib().aaedn_kernel_launches())


def _p(a):
    if a is None:
        return None
    if isinstance(a, int):
        return a
    if hasattr(a, "data_ptr"):
        return a.data_ptr()
    return a.ctypes.data_as(_vp)


# ---------------------------------------------------------------- host tools
def quantize_q4(x):
    """tools/convert_model.py:36-55, bit-exact; returns (codes, fp16 scales)."""
    x = np.ascontiguousarray(x, np.float32).reshape(-1)
    data = np.zeros((x.size + 1) // 2, np.uint8)
    scales = np.zeros((x.size + 31) // 32, np.uint16)
    check(lib().aaedn_quantize_q4(_p(x), x.size, _p(data), _p(scales)))
    return data, scales


def fnv1a32(b, seed=0x811C9DC5):
    b = np.frombuffer(bytes(b), np.uint8)
    return int(lib().aaedn_fnv1a32(_p(b), b.size, seed))


def synth_normal(seed, tensor_id, n, std=0.02):
    out = np.empty(n, np.float32)
    check(lib().aaedn_synth_normal(seed, tensor_id, std, _p(out), n))
    return out


def synth_tokens(seed, stream_id, vocab, n):
    out = np.empty(n, np.uint32)
    check(lib().aaedn_synth_tokens(seed, stream_id, vocab, _p(out), n))
    return out


def rope_table(max_seq, head_dim, theta=10000.0, formula=1):
    c = np.empty(max_seq * (head_dim // 2), np.float32)
    s = np.empty_like(c)
    check(lib().aaedn_rope_table(_p(c), _p(s), max_seq, head_dim, theta, formula))
    return c, s


# ------------------------------------------------------------------ kernels
def dequant_4bit(d_data, d_scales, d_out, n, scale_kind=SCALE_U16INT, stream=None):
    check(lib().aaedn_cu_dequant_4bit(_p(d_data), _p(d_scales), _p(d_out), n, scale_kind, stream))


def fused_matmul(d_in, d_w, d_scales, d_out, M, N, K, lda=None, ldb=None, ldc=None, scale_kind=SCALE_F16,
                 stream=None):
    check(lib().aaedn_cu_fused_matmul(_p(d_in), _p(d_w), _p(d_scales), _p(d_out), M, N, K, lda or K, ldb or K,
                                      ldc or N, scale_kind, stream))


def repack_tiled(codes, scales, N, K):
    """Host repack of row-major quantized weights (aaedn_quantize_q4's codes
    and fp16 scales) into the tile-major layout of the model's engines."""
    codes = np.ascontiguousarray(codes, np.uint8)
    scales = np.ascontiguousarray(scales).view(np.uint16)
    out = np.empty(lib().aaedn_q4_tiled_bytes(N, K), np.uint8)
    check(lib().aaedn_q4_repack_tiled(_p(codes), _p(scales), N, K, _p(out)))
    return out


def fused_matmul_tiled(d_in, d_tiled, d_out, M, N, K, stream=None):
    """fused_matmul on tile-major weights: M == 1 the decode GEMV engine,
    M > 1 the tcgen05 GEMM (dense [M][K] in, [M][N] out)."""
    check(lib().aaedn_cu_fused_matmul_tiled(_p(d_in), _p(d_tiled), _p(d_out), M, N, K, stream))


def f32_matmul(d_in, d_w, d_out, M, N, K, stream=None):
    check(lib().aaedn_cu_f32_matmul(_p(d_in), _p(d_w), _p(d_out), M, N, K, K, K, N, stream))


def rmsnorm(d_in, d_out, d_w, n, eps=1e-6, stream=None):
    check(lib().aaedn_cu_rmsnorm(_p(d_in), _p(d_out), _p(d_w), n, eps, stream))


def rope_apply(d_q, d_k, seq_len, head_dim, d_cos, d_sin, stream=None):
    check(lib().aaedn_cu_rope_apply(_p(d_q), _p(d_k), seq_len, head_dim, _p(d_cos), _p(d_sin), stream))


def attention(d_q, d_k, d_v, segments, d_out, n_heads, head_dim, scale, stream=None):
    segs = np.ascontiguousarray(segments, np.uint32).reshape(-1)
    check(lib().aaedn_cu_attention(_p(d_q), _p(d_k), _p(d_v), _p(segs), segs.size // 2, _p(d_out), n_heads,
                                   head_dim, scale, stream))


FFN_MODEL, FFN_REFERENCE = 0, 1


def ffn_swiglu(d_in, d_out, batch, hidden, ffn, d_gate, d_up, d_down, d_gs, d_us, d_ds, semantics=FFN_MODEL,
               stream=None):
    """include/ffn.hpp ffn_swiglu on device buffers (FFN_MODEL: fp16 block
    scales, silu(g)*u; FFN_REFERENCE: what src/ffn.cpp computes)."""
    check(lib().aaedn_cu_ffn_swiglu(_p(d_in), _p(d_out), batch, hidden, ffn, _p(d_gate), _p(d_up), _p(d_down),
                                    _p(d_gs), _p(d_us), _p(d_ds), semantics, stream))


def sample(d_logits, vocab, temperature, top_p, u, d_token, stream=None):
    """Next token from device logits on the device (docs/mpd.md:539-554;
    src/main.cpp:214-247 is the reference's plain softmax draw): temperature
    (<= 0: greedy), nucleus top_p in
    (0, 1], multinomial draw with the caller's uniform u in [0, 1); the
    token id goes to the uint32 at d_token."""
    check(lib().aaedn_cu_sample(_p(d_logits), int(vocab), float(temperature), float(top_p), float(u), _p(d_token),
                                stream))


def abn_model_config(path, max_seq=4096):
    """The model shape of a whole-model .abn file (aaedn_abn_model_read_header)
    as a config dict, with the caller's context length."""
    h, c = AbnHeader(), ModelConfig()
    check(lib().aaedn_abn_model_read_header(str(path).encode(), ctypes.byref(h), ctypes.byref(c)))
    d = c.as_dict()
    d["max_seq"] = max_seq
    return d


def abn_read(path):
    """Header and payload of an .abn v2 file (quant_load's checks); raises
    AaednError(EFORMAT) when the file is rejected."""
    h = AbnHeader()
    check(lib().aaedn_abn_read_header(str(path).encode(), ctypes.byref(h)))
    n = h.hidden_dim
    data = np.empty(n * n // 2, np.uint8)
    scales = np.empty(n * n // 32, np.uint16)
    check(lib().aaedn_abn_read_payload(str(path).encode(), ctypes.byref(h), _p(data), _p(scales)))
    return h, data, scales


def attention_noalloc(d_q, d_k, d_v, segments, d_out, n_heads, head_dim, scale, stream=None):
    """attention() for callers that cannot allocate device memory: the
    library uses its fixed 1 MiB scratch array instead of allocating, so
    calls that overlap on the GPU race and must be serialised."""
    segs = np.ascontiguousarray(segments, np.uint32).reshape(-1)
    check(lib().aaedn_cu_attention_noalloc(_p(d_q), _p(d_k), _p(d_v), _p(segs), segs.size // 2, _p(d_out), n_heads,
                                           head_dim, scale, stream))


ATTN_NOALLOC_SCRATCH_BYTES = 1 << 20


def device_sync():
    check(lib().aaedn_device_sync())


# -------------------------------------------------------------------- model
TINY = dict(dim=288, n_layers=6, n_heads=6, n_kv_heads=6, head_dim=48, ffn_dim=768, vocab=32000, max_seq=256,
            rope_theta=10000.0, eps=1e-6)
LLAMA2_7B = dict(dim=4096, n_layers=32, n_heads=32, n_kv_heads=32, head_dim=128, ffn_dim=11008, vocab=32000,
                 max_seq=4096, rope_theta=10000.0, eps=1e-6)
LLAMA3_8B = dict(dim=4096, n_layers=32, n_heads=32, n_kv_heads=8, head_dim=128, ffn_dim=14336, vocab=128256,
                 max_seq=4096, rope_theta=500000.0, eps=1e-6)
# the 70B shape of the batched-branch workload (64 query / 8 KV heads, ctx 8192)
LLAMA_70B = dict(dim=8192, n_layers=80, n_heads=64, n_kv_heads=8, head_dim=128, ffn_dim=28672, vocab=128256,
                 max_seq=8192, rope_theta=500000.0, eps=1e-6)

LAYER_MATS = ("wq", "wk", "wv", "wo", "wg", "wu", "wd")


def layer_shapes(cfg):
    D, hd, H, KV, F = cfg["dim"], cfg["head_dim"], cfg["n_heads"], cfg["n_kv_heads"], cfg["ffn_dim"]
    return {"wq": (H * hd, D), "wk": (KV * hd, D), "wv": (KV * hd, D), "wo": (D, H * hd), "wg": (F, D),
            "wu": (F, D), "wd": (D, F)}


def synthetic_weights(cfg, seed):
    """Host weights of the seeded synthetic model in logical layout, the same
    tensors aaedn_model_synthesize uploads: N(0, 0.02) linear weights
    quantized with the block quantizer, fp32 embedding/lm_head, gains 1.0.
    Tensor ids: embedding 0, lm_head 1, layer l: 16 + 8l + index in
    (q, k, v, o, g, u, d)."""
    L, D, V = cfg["n_layers"], cfg["dim"], cfg["vocab"]
    shapes = layer_shapes(cfg)
    w = {k: [] for k in LAYER_MATS}
    w["attn_norm"] = [np.ones(D, np.float32) for _ in range(L)]
    w["ffn_norm"] = [np.ones(D, np.float32) for _ in range(L)]
    for l in range(L):
        for i, name in enumerate(LAYER_MATS):
            r, c = shapes[name]
            x = synth_normal(seed, 16 + 8 * l + i, r * c)
            w[name].append(quantize_q4(x))
    w["embedding"] = synth_normal(seed, 0, V * D).reshape(V, D)
    w["lm_head"] = synth_normal(seed, 1, V * D).reshape(V, D)
    w["final_norm"] = np.ones(D, np.float32)
    return w


TP_HANDLE_BYTES = 64


class Model:
    """One aaedn_model (device arena, weights, paged KV cache, stream).

    tp=(rank, size) makes this process the tensor-parallel rank `rank` of
    `size` (one process per GPU, that GPU current). Every rank then calls
    tp_connect with the handles of all ranks (see connect_tp) before its
    first step, and all ranks run the same calls with the same tokens."""

    def __init__(self, cfg, tp=None):
        self.cfg = dict(cfg)
        c = ModelConfig(**{k: self.cfg[k] for k, _ in ModelConfig._fields_})
        h = _vp()
        if tp is None or tp[1] == 1:
            check(lib().aaedn_model_create(ctypes.byref(c), ctypes.byref(h)))
            self.tp = (0, 1)
        else:
            check(lib().aaedn_model_create_tp(ctypes.byref(c), int(tp[0]), int(tp[1]), ctypes.byref(h)))
            self.tp = (int(tp[0]), int(tp[1]))
        self.h = h

    def tp_handle(self):
        """This rank's peer handle (bytes) for the other ranks."""
        out = np.zeros(TP_HANDLE_BYTES, np.uint8)
        check(lib().aaedn_model_tp_handle(self.h, _p(out)))
        return out.tobytes()

    def tp_connect(self, handles):
        """handles: the tp_handle() bytes of every rank, in rank order."""
        buf = np.frombuffer(b"".join(handles), np.uint8).copy()
        check(lib().aaedn_model_tp_connect(self.h, _p(buf)))

    def connect_tp(self, group=None):
        """Exchanges handles over torch.distributed and connects."""
        import torch.distributed as dist
        hs = [None] * self.tp[1]
        dist.all_gather_object(hs, self.tp_handle(), group=group)
        self.tp_connect(hs)

    def tp_share(self):
        """(first token id, count) of this rank's lm_head rows / logits slice."""
        p = tp_plan(self.cfg, self.tp[0], self.tp[1])
        return p["vocab0"], p["vocab"]

    def next_token(self):
        """The greedy token of the last step (synchronises)."""
        t = _u32()
        check(lib().aaedn_model_next_token(self.h, ctypes.byref(t)))
        return int(t.value)

    def status(self):
        """Raises if a bounded device wait ran out or a position passed the
        cache (synchronises)."""
        check(lib().aaedn_model_status(self.h))

    def close(self):
        if getattr(self, "h", None):
            lib().aaedn_model_destroy(self.h)
            self.h = None

    __del__ = close

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    @property
    def stream(self):
        return lib().aaedn_model_stream(self.h)

    @property
    def arena_bytes(self):
        return int(lib().aaedn_model_arena_bytes(self.h))

    @property
    def pos(self):
        return int(lib().aaedn_model_pos(self.h))

    @property
    def kernels_per_step(self):
        return int(lib().aaedn_model_kernels_per_step(self.h))

    @property
    def prefill_rows(self):
        """Prompt tokens per tensor-core prefill chunk (0: one decode step per
        prompt token)."""
        return int(lib().aaedn_model_prefill_rows(self.h))

    def set_weights(self, w):
        keep = []
        for l in range(self.cfg["n_layers"]):
            lh = LayerHost()
            for name in LAYER_MATS:
                d, s = w[name][l]
                d = np.ascontiguousarray(d)
                s = np.ascontiguousarray(s)
                keep += [d, s]
                setattr(lh, name, _p(d))
                setattr(lh, "s" + name[1], _p(s))
            an = np.ascontiguousarray(w["attn_norm"][l], np.float32)
            fn = np.ascontiguousarray(w["ffn_norm"][l], np.float32)
            keep += [an, fn]
            lh.attn_norm, lh.ffn_norm = _p(an), _p(fn)
            check(lib().aaedn_model_set_layer(self.h, l, ctypes.byref(lh)))
        emb = np.ascontiguousarray(w["embedding"], np.float32)
        fnorm = np.ascontiguousarray(w["final_norm"], np.float32)
        lm = np.ascontiguousarray(w["lm_head"], np.float32)
        check(lib().aaedn_model_set_globals(self.h, _p(emb), _p(fnorm), _p(lm)))

    def synthesize(self, seed):
        check(lib().aaedn_model_synthesize(self.h, seed))

    def load_abn(self, path):
        """Every weight from a whole-model .abn file of this model's shape."""
        check(lib().aaedn_model_load_abn(self.h, str(path).encode()))

    def reset(self):
        check(lib().aaedn_model_reset(self.h))

    def forward(self, tokens, want_logits=True, out=None):
        """transformer_forward: the logits of the last token (out: a host
        float32 array of vocab entries to fill, e.g. pinned memory; else a
        new array)."""
        t = np.ascontiguousarray(tokens, np.uint32).reshape(-1)
        if out is not None:
            if out.dtype != np.float32 or out.size != self.cfg["vocab"] or not out.flags["C_CONTIGUOUS"]:
                raise ValueError("out must be a contiguous float32 array of vocab entries")
            logits = out
        else:
            logits = np.empty(self.cfg["vocab"], np.float32) if want_logits else None
        check(lib().aaedn_model_forward(self.h, _p(t), t.size, _p(logits)))
        return logits

    def generate(self, prompt, n_new):
        p = np.ascontiguousarray(prompt, np.uint32).reshape(-1)
        out = np.empty(n_new, np.uint32)
        check(lib().aaedn_model_generate(self.h, _p(p), p.size, n_new, _p(out)))
        return out

    def decode_steps(self, n):
        check(lib().aaedn_model_decode_steps(self.h, n))

    def logits(self):
        out = np.empty(self.cfg["vocab"], np.float32)
        check(lib().aaedn_model_logits(self.h, _p(out)))
        return out

    def tokens(self, n):
        out = np.empty(n, np.uint32)
        check(lib().aaedn_model_tokens(self.h, _p(out), n))
        return out

    def rewind(self, pos):
        check(lib().aaedn_model_rewind(self.h, pos))

    def profile_step(self):
        """Device ms of every kernel of one decode step (launch order)."""
        n = self.kernels_per_step
        out = np.empty(n, np.float32)
        got = _u32()
        check(lib().aaedn_model_profile_step(self.h, _p(out), n, ctypes.byref(got)))
        return out[:got.value]

    PART_NAMES = ("step", "gemv", "qkv", "attention", "o", "gate_up", "down", "lm_head")

    def profile_parts(self, reps=10):
        """ms per step of sub-graphs of the decode step (tracing)."""
        out = np.empty(8, np.float32)
        check(lib().aaedn_model_profile_parts(self.h, reps, _p(out), 8))
        return dict(zip(self.PART_NAMES, out.tolist()))

    def trace_kernels(self):
        """globaltimer stamps (ns) of one decode step of the per-kernel graph:
        (stamps [5 * n_layers + 1][1024][4], grid [5 * n_layers + 1]); per
        launch and CTA: entry, operand ready, first weights, exit."""
        nk = self.cfg["n_layers"] * 5 + 1
        st = np.zeros(nk * 1024 * 4, np.uint64)
        grid = np.zeros(nk, np.uint32)
        check(lib().aaedn_model_trace_kernels(self.h, _p(st), st.size, _p(grid), grid.size))
        return st.reshape(nk, 1024, 4), grid

    def forward_debug(self, token):
        hidden = np.empty((self.cfg["n_layers"], self.cfg["dim"]), np.float32)
        logits = np.empty(self.cfg["vocab"], np.float32)
        check(lib().aaedn_model_forward_debug(self.h, int(token), _p(hidden), _p(logits)))
        return hidden, logits


class BatchedModel(Model):
    """A model holding up to max_seqs sequences over one pool of KV pages
    (kv_tokens cached tokens in all): open / fork / close sequences, prefill
    one, step many at once (aaedn_model_create_batched)."""

    def __init__(self, cfg, max_seqs, kv_tokens):
        self.cfg = dict(cfg)
        c = ModelConfig(**{k: self.cfg[k] for k, _ in ModelConfig._fields_})
        h = _vp()
        check(lib().aaedn_model_create_batched(ctypes.byref(c), int(max_seqs), int(kv_tokens), ctypes.byref(h)))
        self.tp = (0, 1)
        self.h = h
        self.max_seqs = int(max_seqs)

    def open(self):
        s = _u32()
        check(lib().aaedn_seq_open(self.h, ctypes.byref(s)))
        return int(s.value)

    def fork(self, parent):
        s = _u32()
        check(lib().aaedn_seq_fork(self.h, int(parent), ctypes.byref(s)))
        return int(s.value)

    def close_seq(self, seq):
        check(lib().aaedn_seq_close(self.h, int(seq)))

    def seq_len(self, seq):
        n = _u32()
        check(lib().aaedn_seq_len(self.h, int(seq), ctypes.byref(n)))
        return int(n.value)

    def kv_pages(self):
        """(pages in the pool, free pages)."""
        t, f = _u32(), _u32()
        check(lib().aaedn_model_kv_pages(self.h, ctypes.byref(t), ctypes.byref(f)))
        return int(t.value), int(f.value)

    def prefill(self, seq, tokens, want_logits=True):
        """Appends tokens to one sequence; (last logits or None, greedy next)."""
        t = np.ascontiguousarray(tokens, np.uint32).reshape(-1)
        logits = np.empty(self.cfg["vocab"], np.float32) if want_logits else None
        nxt = np.zeros(1, np.uint32)
        check(lib().aaedn_seq_prefill(self.h, int(seq), _p(t), t.size, _p(logits), _p(nxt)))
        return logits, int(nxt[0])

    def step(self, seqs, tokens, want_logits=True):
        """One token for each sequence; (logits [n][vocab] or None, greedy next [n])."""
        sq = np.ascontiguousarray(seqs, np.uint32).reshape(-1)
        t = np.ascontiguousarray(tokens, np.uint32).reshape(-1)
        logits = np.empty((sq.size, self.cfg["vocab"]), np.float32) if want_logits else None
        nxt = np.zeros(sq.size, np.uint32)
        check(lib().aaedn_model_step_batch(self.h, _p(sq), _p(t), sq.size, _p(logits), _p(nxt)))
        return logits, nxt
