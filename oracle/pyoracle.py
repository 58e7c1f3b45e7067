"""ctypes wrapper over oracle/build/liboracle*.so.

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and
bench.py's cpu_baseline leg as the checker / the timed CPU restatement.
The product library never imports this module.
"""
import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))

_vp = ctypes.c_void_p
_sz = ctypes.c_size_t
_u32 = ctypes.c_uint32


def build(quiet=True):
    """Compile the oracle (and oracle/_ref when the reference checkout exists)."""
    out = subprocess.run(["make", "-C", HERE], capture_output=True, text=True)
    if out.returncode != 0:
        raise RuntimeError("oracle build failed:\n" + out.stdout + out.stderr)
    if not quiet:
        print(out.stdout)


def ptr(a):
    return None if a is None else a.ctypes.data_as(_vp)


class OrConfig(ctypes.Structure):
    _fields_ = [("dim", _u32), ("n_layers", _u32), ("n_heads", _u32), ("n_kv_heads", _u32),
                ("head_dim", _u32), ("ffn_dim", _u32), ("vocab", _u32), ("max_seq", _u32),
                ("rope_theta", ctypes.c_double), ("eps", ctypes.c_float)]


class OrQ4(ctypes.Structure):
    _fields_ = [("data", _vp), ("scales", _vp)]


class OrWeights(ctypes.Structure):
    _fields_ = [("embedding", _vp), ("final_norm", _vp), ("lm_head", _vp),
                ("attn_norm", ctypes.POINTER(_vp)), ("ffn_norm", ctypes.POINTER(_vp)),
                ("wq", ctypes.POINTER(OrQ4)), ("wk", ctypes.POINTER(OrQ4)), ("wv", ctypes.POINTER(OrQ4)),
                ("wo", ctypes.POINTER(OrQ4)), ("wg", ctypes.POINTER(OrQ4)), ("wu", ctypes.POINTER(OrQ4)),
                ("wd", ctypes.POINTER(OrQ4))]


class Oracle:
    """One of the two oracle builds: strict (parity) or fast (timed baseline)."""

    def __init__(self, fast=False):
        self.fast = bool(fast)
        name = "liboracle_fast.so" if fast else "liboracle.so"
        path = os.path.join(HERE, "build", name)
        if not os.path.exists(path):
            build()
        L = ctypes.CDLL(path)
        self.lib = L
        L.or_f16_to_f32.argtypes = [ctypes.c_uint16]
        L.or_f16_to_f32.restype = ctypes.c_float
        L.or_f64_to_f16.argtypes = [ctypes.c_double]
        L.or_f64_to_f16.restype = ctypes.c_uint16
        L.or_quantize_q4.argtypes = [_vp, _sz, _vp, _vp]
        L.or_dequant_4bit.argtypes = [_vp, _vp, _vp, _sz]
        L.or_dequant_4bit_f16.argtypes = [_vp, _vp, _vp, _sz]
        L.or_q4_matmul.argtypes = [_vp, _vp, _vp, _vp, _sz, _sz, _sz, _sz, _sz, _sz, ctypes.c_int]
        L.or_f32_matmul.argtypes = [_vp, _vp, _vp, _sz, _sz, _sz, _sz, _sz, _sz]
        L.or_rmsnorm.argtypes = [_vp, _vp, _vp, _sz, ctypes.c_float]
        L.or_rope_tables_ref.argtypes = [_vp, _vp, _sz, _sz]
        L.or_rope_tables.argtypes = [_vp, _vp, _sz, _sz, ctypes.c_double]
        L.or_rope_apply.argtypes = [_vp, _vp, _sz, _sz, _vp, _vp]
        L.or_attention.argtypes = [_vp, _vp, _vp, _vp, _sz, _vp, _sz, _sz, ctypes.c_float]
        L.or_ffn_swiglu_refsem.argtypes = [_vp, _vp, _sz, _sz, _sz, _vp, _vp, _vp, _vp, _vp, _vp]
        L.or_fnv1a32.argtypes = [_vp, _sz, _u32]
        L.or_fnv1a32.restype = _u32
        L.or_abn_v2_accepts.argtypes = [_vp, _sz]
        L.or_abn_v2_accepts.restype = ctypes.c_int
        L.or_model_create.argtypes = [ctypes.POINTER(OrConfig), ctypes.POINTER(OrWeights)]
        L.or_model_create.restype = _vp
        L.or_model_destroy.argtypes = [_vp]
        L.or_model_reset.argtypes = [_vp]
        L.or_model_pos.argtypes = [_vp]
        L.or_model_pos.restype = _u32
        L.or_model_step.argtypes = [_vp, _u32, _vp, _vp]
        L.or_model_step.restype = ctypes.c_int
        L.or_argmax.argtypes = [_vp, _sz]
        L.or_argmax.restype = _u32
        L.or_model_generate.argtypes = [_vp, _vp, _sz, _sz, _vp, _vp]
        L.or_model_generate.restype = ctypes.c_int
        L.or_set_threads.argtypes = [ctypes.c_int]
        L.or_get_threads.restype = ctypes.c_int
        L.or_synth_normal.argtypes = [ctypes.c_uint64, ctypes.c_uint64, ctypes.c_float, _vp, _sz]
        L.or_synth_tokens.argtypes = [ctypes.c_uint64, ctypes.c_uint64, _u32, _vp, _sz]
        L.or_model_seek.argtypes = [_vp, _u32]
        L.or_model_seek.restype = ctypes.c_int

    # -- primitives -------------------------------------------------------
    def quantize(self, x):
        x = np.ascontiguousarray(x, np.float32).reshape(-1)
        n = x.size
        data = np.zeros((n + 1) // 2, np.uint8)
        scales = np.zeros((n + 31) // 32, np.uint16)
        self.lib.or_quantize_q4(ptr(x), n, ptr(data), ptr(scales))
        return data, scales

    def dequant(self, data, scales, n, f16=False):
        out = np.empty(n, np.float32)
        f = self.lib.or_dequant_4bit_f16 if f16 else self.lib.or_dequant_4bit
        f(ptr(data), ptr(scales), ptr(out), n)
        return out

    def q4_matmul(self, x, data, scales, N, K, scale_kind=0, ldb=None):
        x = np.ascontiguousarray(x, np.float32)
        M = x.shape[0] if x.ndim == 2 else 1
        lda = x.shape[-1]
        out = np.empty((M, N), np.float32)
        self.lib.or_q4_matmul(ptr(x), ptr(data), ptr(scales), ptr(out), M, N, K, lda, ldb or K, N, scale_kind)
        return out

    def f32_matmul(self, x, w):
        x = np.ascontiguousarray(x, np.float32)
        M = x.shape[0] if x.ndim == 2 else 1
        N, K = w.shape
        out = np.empty((M, N), np.float32)
        self.lib.or_f32_matmul(ptr(x), ptr(w), ptr(out), M, N, K, K, K, N)
        return out

    def rmsnorm(self, x, w, eps=1e-6):
        x = np.ascontiguousarray(x, np.float32)
        out = np.empty_like(x)
        self.lib.or_rmsnorm(ptr(x), ptr(out), ptr(np.ascontiguousarray(w, np.float32)), x.size, eps)
        return out

    def rope_tables_ref(self, max_seq, hd):
        c = np.empty(max_seq * (hd // 2), np.float32)
        s = np.empty_like(c)
        self.lib.or_rope_tables_ref(ptr(c), ptr(s), max_seq, hd)
        return c, s

    def rope_tables(self, max_seq, hd, theta):
        c = np.empty(max_seq * (hd // 2), np.float32)
        s = np.empty_like(c)
        self.lib.or_rope_tables(ptr(c), ptr(s), max_seq, hd, theta)
        return c, s

    def rope_apply(self, q, k, seq_len, hd, c, s):
        q = np.array(q, np.float32)
        k = np.array(k, np.float32)
        self.lib.or_rope_apply(ptr(q), ptr(k), seq_len, hd, ptr(c), ptr(s))
        return q, k

    def attention(self, q, kc, vc, segs, n_heads, hd, scale):
        out = np.empty(n_heads * hd, np.float32)
        segs = np.ascontiguousarray(segs, np.uint32)
        self.lib.or_attention(ptr(q), ptr(kc), ptr(vc), ptr(segs), segs.size // 2, ptr(out), n_heads, hd, scale)
        return out

    def fnv1a32(self, b):
        b = np.frombuffer(bytes(b), np.uint8)
        return self.lib.or_fnv1a32(ptr(b), b.size, 0x811C9DC5)

    def abn_v2_accepts(self, blob):
        b = np.frombuffer(bytes(blob), np.uint8)
        return bool(self.lib.or_abn_v2_accepts(ptr(b), b.size))

    def synth_normal(self, seed, tensor_id, n, std=0.02):
        out = np.empty(n, np.float32)
        self.lib.or_synth_normal(seed, tensor_id, std, ptr(out), n)
        return out

    def synth_tokens(self, seed, stream_id, vocab, n):
        out = np.empty(n, np.uint32)
        self.lib.or_synth_tokens(seed, stream_id, vocab, ptr(out), n)
        return out

    def set_threads(self, n):
        self.lib.or_set_threads(int(n))

    def threads(self):
        return self.lib.or_get_threads()


LAYER_MATS = ("wq", "wk", "wv", "wo", "wg", "wu", "wd")


def layer_shapes(cfg):
    D, hd, H, KV, F = cfg["dim"], cfg["head_dim"], cfg["n_heads"], cfg["n_kv_heads"], cfg["ffn_dim"]
    return {"wq": (H * hd, D), "wk": (KV * hd, D), "wv": (KV * hd, D), "wo": (D, H * hd), "wg": (F, D),
            "wu": (F, D), "wd": (D, F)}


def synthetic_weights(cfg, seed, oracle=None):
    """The seeded synthetic model built on the oracle side alone: the same
    tensors as the library's synthetic model (tensor ids: embedding 0,
    lm_head 1, layer l: 16 + 8l + index in (q, k, v, o, g, u, d); N(0, 0.02)
    linear weights quantized with the oracle's restatement of
    tools/convert_model.py:36-55; fp32 embedding/lm_head; gains 1.0). The
    strict build generates and quantizes (bit-exact with the library)."""
    o = oracle if (oracle is not None and not getattr(oracle, "fast", False)) else Oracle()
    L, D, V = cfg["n_layers"], cfg["dim"], cfg["vocab"]
    shapes = layer_shapes(cfg)
    w = {k: [] for k in LAYER_MATS}
    w["attn_norm"] = [np.ones(D, np.float32) for _ in range(L)]
    w["ffn_norm"] = [np.ones(D, np.float32) for _ in range(L)]
    for l in range(L):
        for i, name in enumerate(LAYER_MATS):
            r, c = shapes[name]
            w[name].append(o.quantize(o.synth_normal(seed, 16 + 8 * l + i, r * c)))
    w["embedding"] = o.synth_normal(seed, 0, V * D).reshape(V, D)
    w["lm_head"] = o.synth_normal(seed, 1, V * D).reshape(V, D)
    w["final_norm"] = np.ones(D, np.float32)
    return w


def synth_tokens(seed, stream_id, vocab, n):
    """The library's seeded prompt ids, from the oracle's restatement."""
    return Oracle().synth_tokens(seed, stream_id, vocab, n)


class OracleModel:
    """The model oracle over host weights (a dict as produced by the
    synthetic generator: per-layer lists of (data, scales) and fp32 arrays)."""

    def __init__(self, oracle, cfg, w):
        self.o = oracle
        self.cfg = cfg
        L = cfg["n_layers"]
        self._keep = [w]
        c = OrConfig(cfg["dim"], L, cfg["n_heads"], cfg["n_kv_heads"], cfg["head_dim"], cfg["ffn_dim"],
                     cfg["vocab"], cfg["max_seq"], float(cfg["rope_theta"]), float(cfg.get("eps", 1e-6)))

        def q4arr(name):
            arr = (OrQ4 * L)()
            for l in range(L):
                d, s = w[name][l]
                arr[l] = OrQ4(ptr(d), ptr(s))
            self._keep.append(arr)
            return arr

        def farr(name):
            arr = (_vp * L)()
            for l in range(L):
                arr[l] = ptr(w[name][l])
            self._keep.append(arr)
            return arr

        ws = OrWeights(ptr(w["embedding"]), ptr(w["final_norm"]), ptr(w["lm_head"]), farr("attn_norm"),
                       farr("ffn_norm"), q4arr("wq"), q4arr("wk"), q4arr("wv"), q4arr("wo"), q4arr("wg"),
                       q4arr("wu"), q4arr("wd"))
        self._keep.append(ws)
        self._cfg = c
        self.h = oracle.lib.or_model_create(ctypes.byref(c), ctypes.byref(ws))
        if not self.h:
            raise MemoryError("or_model_create failed")

    def __del__(self):
        if getattr(self, "h", None):
            self.o.lib.or_model_destroy(self.h)
            self.h = None

    def reset(self):
        self.o.lib.or_model_reset(self.h)

    @property
    def pos(self):
        return self.o.lib.or_model_pos(self.h)

    def seek(self, pos):
        """Timing aid: jump to position pos with synthetic cached K/V rows."""
        if self.o.lib.or_model_seek(self.h, int(pos)) != 0:
            raise ValueError(f"seek to {pos} outside the cache")

    def step(self, token, want_hidden=False):
        logits = np.empty(self.cfg["vocab"], np.float32)
        hidden = np.empty((self.cfg["n_layers"], self.cfg["dim"]), np.float32) if want_hidden else None
        rc = self.o.lib.or_model_step(self.h, int(token), ptr(logits), ptr(hidden))
        if rc != 0:
            raise RuntimeError("or_model_step failed")
        return (logits, hidden) if want_hidden else logits

    def generate(self, prompt, n_new):
        prompt = np.ascontiguousarray(prompt, np.uint32)
        out = np.empty(n_new, np.uint32)
        logits = np.empty(self.cfg["vocab"], np.float32)
        rc = self.o.lib.or_model_generate(self.h, ptr(prompt), prompt.size, n_new, ptr(out), ptr(logits))
        if rc != 0:
            raise RuntimeError("or_model_generate failed")
        return out, logits


def sample_ref(logits, temperature, top_p, u):
    """Next-token sampling as the reference specifies it (docs/mpd.md:539-554),
    sorting explicitly (src/main.cpp:214-247, the reference's plain softmax
    draw, walks ids in index order instead; sample_main_ref restates it): temperature <= 0 is the argmax (ties to the lowest id);
    otherwise p = exp((l - max) * (1/T)) in fp32, tokens sorted by p
    descending (stable: lower id first), kept up to and including the first
    whose cumulative sum reaches top_p * sum(p), then the first kept token
    whose cumulative sum reaches u times the kept mass. Cumulative sums in
    fp64. Returns (token, margin): margin is the smallest relative distance
    of a threshold from a cumulative sum it was compared with (decisions
    closer than fp32 rounding of p can differ between implementations)."""
    lg = np.asarray(logits, np.float32)
    if not temperature > 0:
        return int(np.argmax(lg)), np.inf
    mx = lg.max()
    inv_t = np.float32(1.0) / np.float32(temperature)
    p = np.exp((lg - mx) * inv_t).astype(np.float32)
    order = np.argsort(-p, kind="stable")
    cs = np.cumsum(p[order].astype(np.float64))
    z = cs[-1]
    t1 = float(top_p) * z
    k = int(np.searchsorted(cs, t1, side="left"))
    k = min(k, cs.size - 1)  # rounding can leave t1 above the total: keep all
    w = cs[k]
    t2 = float(u) * w
    j = int(np.searchsorted(cs, t2, side="left"))
    margin = np.inf
    for t, i in ((t1, k), (t2, j)):
        for c in (cs[i], cs[i - 1] if i > 0 else None):
            if c is not None and t > 0:
                margin = min(margin, abs(c - t) / t)
    return int(order[j]), margin


def sample_main_ref(logits, r):
    """src/main.cpp:216-246 as written: softmax in fp32 (expf(l - max), sum,
    divide), then the first id whose running fp32 sum reaches r."""
    lg = np.asarray(logits, np.float32)
    e = np.exp(lg - lg.max()).astype(np.float32)
    s = np.float32(0)
    for v in e:
        s = np.float32(s + v)
    pr = (e / s).astype(np.float32)
    c = np.float32(0)
    for i, v in enumerate(pr):
        c = np.float32(c + v)
        if r <= c:
            return i
    return 0
