"""The .abt v2 tokenizer through the C ABI (aaedn_tokenizer_*), and the
.abt writer.

Mirrors the reference's include/tokenizer.hpp (tokenizer_load, encode,
decode; src/tokenizer.cpp:32-257) and its converter
tools/convert_tokenizer.py:44-93 (the payload layout and the header
"<8sIQI4I24s"). Host code only: no GPU is needed.
"""
import ctypes
import struct

import numpy as np

from . import _p, check, fnv1a32, lib

TOKEN_BOS, TOKEN_EOS, TOKEN_PAD = 32765, 32766, 32767
ABT_MAGIC, ABT_VERSION = b"AAEDNTOK", 2


class Tokenizer:
    """A loaded .abt tokenizer (raises AaednError with AAEDN_EFORMAT when the
    file is one the reference rejects)."""

    def __init__(self, path=None, data=None):
        h = ctypes.c_void_p()
        if data is not None:
            buf = np.frombuffer(bytes(data), np.uint8)
            check(lib().aaedn_tokenizer_from_bytes(_p(buf) if buf.size else None, buf.size, ctypes.byref(h)))
        else:
            check(lib().aaedn_tokenizer_load(str(path).encode(), ctypes.byref(h)))
        self._h = h
        info = np.zeros(5, np.uint32)
        check(lib().aaedn_tokenizer_info(self._h, _p(info)))
        (self.vocab_size, self.merge_count, self.max_token_bytes, self.format_version,
         self.payload_checksum) = (int(v) for v in info)

    def close(self):
        if self._h:
            lib().aaedn_tokenizer_free(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def encode(self, text, add_bos=False):
        """Token ids of text (str: UTF-8 bytes; bytes as given, up to the
        first NUL)."""
        b = text.encode() if isinstance(text, str) else bytes(text)
        out = np.empty(len(b) + 1, np.uint32)
        n = ctypes.c_size_t()
        check(lib().aaedn_tokenizer_encode(self._h, b, int(add_bos), _p(out), out.size, ctypes.byref(n)))
        return out[:n.value].copy()

    def decode(self, ids):
        """The bytes of the ids' strings, concatenated."""
        ids = np.ascontiguousarray(ids, np.uint32)
        n = ctypes.c_size_t()
        check(lib().aaedn_tokenizer_decode(self._h, _p(ids) if ids.size else None, ids.size, None, 0,
                                           ctypes.byref(n)))
        buf = ctypes.create_string_buffer(n.value + 1)
        check(lib().aaedn_tokenizer_decode(self._h, _p(ids) if ids.size else None, ids.size, buf, n.value + 1,
                                           ctypes.byref(n)))
        return buf.raw[:n.value]


def abt_bytes(tokens, merges, max_token_bytes=None):
    """An .abt v2 file image: tokens = the token strings (bytes or str) in id
    order, merges = (first id, second id) rules in rule order."""
    toks = [t.encode("utf-8") if isinstance(t, str) else bytes(t) for t in tokens]
    strings, offsets = bytearray(), []
    for t in toks:
        offsets.append(len(strings))
        strings += t + b"\0"
    mtb = max((len(t) for t in toks), default=0) if max_token_bytes is None else max_token_bytes
    payload = bytearray(struct.pack("<IIII", len(toks), mtb, len(merges), len(strings)))
    payload += strings
    payload += struct.pack(f"<{len(offsets)}I", *offsets)
    for a, b in merges:
        payload += struct.pack("<HH", a & 0xFFFF, b & 0xFFFF)
    header = struct.pack("<8sIQI4I24s", ABT_MAGIC, ABT_VERSION, len(payload), fnv1a32(bytes(payload)), len(toks),
                         mtb, len(merges), len(payload), b"\0" * 24)
    return header + bytes(payload)


def write_abt(path, tokens, merges):
    with open(path, "wb") as f:
        f.write(abt_bytes(tokens, merges))


def from_hf(tokenizer):
    """(tokens, merges) of a Hugging Face tokenizer object, as the
    reference's converter reads them: the vocabulary sorted by id, the merge
    strings split at a space (else at '##'), unknown halves as id 0, ids
    kept to 16 bits."""
    vocab = tokenizer.get_vocab()
    tokens = [t for t, _ in sorted(vocab.items(), key=lambda kv: kv[1])]
    merges = []
    for m in getattr(tokenizer, "merges", None) or []:
        if not isinstance(m, str):
            continue
        parts = m.split(" ")
        if len(parts) != 2:
            parts = m.split("##")
        if len(parts) != 2:
            continue
        merges.append((int(vocab.get(parts[0], 0)) & 0xFFFF, int(vocab.get(parts[1], 0)) & 0xFFFF))
    return tokens, merges
