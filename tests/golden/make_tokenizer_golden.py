#!/usr/bin/env python3
"""Generate tokenizer_golden.npz: the reference tokenizer's own answers
(src/tokenizer.cpp, compiled from source into oracle/_ref/libaaedn_ref.so by
``make -C oracle AAEDN_REF=...``) on seeded .abt files and texts.

* two tokenizers: a seeded one (256 byte tokens, 200 longer strings, 400
  rules over bytes and over earlier merged ids, with repeated-letter rules
  whose overlapping pairs tie in the queue and duplicate rules) and the
  two-token fixture of tests/test_artifact_roundtrip.cpp;
* texts: empty, single bytes, runs of one letter, random strings over a small
  alphabet (many merges and ties), all bytes 1..255, UTF-8 text; encoded with
  and without BOS, and decoded back;
* decodes of id lists with BOS, EOS, PAD, merged and out-of-range ids;
* the loader's accept/reject decision on corrupted and edge-case images.

Run where the reference checkout exists (AAEDN_REF). The fixture is
committed; tests read only the fixture.
"""
import ctypes
import os
import struct
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
REF = os.environ.get("AAEDN_REF")


def fnv1a32(data, h=0x811C9DC5):
    for b in data:
        h ^= b
        h = (h * 0x01000193) & 0xFFFFFFFF
    return h


def abt(tokens, merges, max_bytes=None, version=2, magic=b"AAEDNTOK", counts=None, block=None, extra=b"",
        checksum=None, declared=None, size=None):
    """An .abt image, each field overridable to build rejected files."""
    strings, offs = bytearray(), []
    for t in tokens:
        offs.append(len(strings))
        strings += t + b"\0"
    mb = max((len(t) for t in tokens), default=0) if max_bytes is None else max_bytes
    v, m = len(tokens), len(merges)
    pc = counts or (v, mb, m)
    payload = bytearray(struct.pack("<IIII", pc[0], pc[1], pc[2], len(strings) if block is None else block))
    payload += strings
    payload += struct.pack(f"<{v}I", *offs)
    for a, b in merges:
        payload += struct.pack("<HH", a, b)
    payload += extra
    ps = len(payload) if size is None else size
    hdr = struct.pack("<8sIQI4I24s", magic, version, ps, fnv1a32(payload) if checksum is None else checksum, v, mb, m,
                      ps if declared is None else declared, b"\0" * 24)
    return hdr + bytes(payload)


def seeded_tokenizer(rng):
    tokens = [bytes([i]) for i in range(256)]
    alpha = b"abcdefgh xyz"
    for _ in range(200):
        n = int(rng.integers(2, 7))
        tokens.append(bytes(alpha[int(k)] for k in rng.integers(0, len(alpha), n)))
    vocab = len(tokens)
    merges = []
    for c in b"abcxa":  # repeated letters: overlapping pairs that tie
        merges.append((c, c))
    while len(merges) < 400:
        r = rng.random()
        if r < 0.6:
            a, b = (int(alpha[int(k)]) for k in rng.integers(0, len(alpha), 2))
        elif r < 0.9 and merges:
            a = vocab + int(rng.integers(0, len(merges)))  # an earlier rule's merged id
            b = int(alpha[int(rng.integers(0, len(alpha)))])
        else:
            a, b = merges[int(rng.integers(0, len(merges)))]  # a duplicate rule
        merges.append((a, b))
    return tokens, merges


def texts(rng):
    out = [b"", b"a", b"aa", b"aaa", b"aaaaaaa", b"ab", b"abababab", b"xaxaxa", b"hello world",
           bytes(range(1, 256)), "naïve café — 東京".encode()]
    alpha = b"abcdefgh xyz"
    for _ in range(40):
        n = int(rng.integers(1, 160))
        out.append(bytes(alpha[int(k)] for k in rng.integers(0, len(alpha), n)))
    for _ in range(8):
        out.append(bytes(int(k) for k in rng.integers(1, 256, int(rng.integers(1, 64)))))
    return out


def load_ref():
    lib = ctypes.CDLL(os.path.join(REPO, "oracle", "_ref", "libaaedn_ref.so"))
    vp, sz = ctypes.c_void_p, ctypes.c_size_t
    lib.ref_tokenizer.argtypes = [ctypes.c_char_p, ctypes.c_char_p, ctypes.c_int, vp, vp, sz,
                                  ctypes.POINTER(sz), vp, sz, ctypes.POINTER(sz)]
    lib.ref_tokenizer.restype = ctypes.c_int
    lib.ref_tokenizer_decode.argtypes = [ctypes.c_char_p, vp, sz, vp, sz]
    lib.ref_tokenizer_decode.restype = sz
    return lib


def ref_run(lib, path, text, add_bos):
    info = np.zeros(5, np.uint32)
    n = len(text) if text is not None else 0
    ids = np.zeros(n + 2, np.uint32)
    buf = ctypes.create_string_buffer(4 * n + 64)
    ni, nb = ctypes.c_size_t(), ctypes.c_size_t()
    ok = lib.ref_tokenizer(path.encode(), text, add_bos, info.ctypes.data, ids.ctypes.data, ids.size,
                           ctypes.byref(ni), buf, len(buf), ctypes.byref(nb))
    return ok, info, ids[:ni.value].copy(), buf.raw[:nb.value]


def main():
    if not REF or not os.path.isdir(os.path.join(REF, "src")):
        raise SystemExit("set AAEDN_REF to the reference project's root (the directory holding src/)")
    lib = load_ref()
    rng = np.random.default_rng(20261202)
    out = {}
    tmp = tempfile.mkdtemp()
    toks, merges = seeded_tokenizer(rng)
    tok_imgs = {"seeded": abt(toks, merges), "roundtrip": abt([b"a", b"b"], [(0, 1)])}
    tx = texts(rng)
    out["text_bytes"] = np.frombuffer(b"".join(tx), np.uint8)
    out["text_len"] = np.array([len(t) for t in tx], np.int64)
    for name, img in tok_imgs.items():
        out[f"tok_{name}"] = np.frombuffer(img, np.uint8)
        path = os.path.join(tmp, name + ".abt")
        with open(path, "wb") as f:
            f.write(img)
        for bos in (0, 1):
            all_ids, n_ids, all_dec, n_dec = [], [], [], []
            for t in tx:
                ok, info, ids, dec = ref_run(lib, path, t, bos)
                assert ok
                all_ids.append(ids)
                n_ids.append(ids.size)
                all_dec.append(dec)
                n_dec.append(len(dec))
            out[f"{name}_bos{bos}_ids"] = np.concatenate(all_ids).astype(np.uint32)
            out[f"{name}_bos{bos}_n"] = np.array(n_ids, np.int64)
            out[f"{name}_bos{bos}_dec"] = np.frombuffer(b"".join(all_dec), np.uint8)
            out[f"{name}_bos{bos}_dec_n"] = np.array(n_dec, np.int64)
        out[f"{name}_info"] = info
        # decodes of arbitrary id lists
        vocab = int(info[0])
        lists = [[32765, 32766, 32767], [0, 1, vocab - 1, vocab, vocab + 5, 1 << 20], list(range(min(vocab, 300)))]
        for _ in range(5):
            lists.append([int(k) for k in rng.integers(0, vocab + 50, int(rng.integers(1, 40)))])
        dec, dn, ids_cat, ids_n = [], [], [], []
        for L in lists:
            a = np.array(L, np.uint32)
            buf = ctypes.create_string_buffer(1 << 16)
            n = lib.ref_tokenizer_decode(path.encode(), a.ctypes.data, a.size, buf, len(buf))
            dec.append(buf.raw[:n])
            dn.append(n)
            ids_cat.append(a)
            ids_n.append(a.size)
        out[f"{name}_declist_ids"] = np.concatenate(ids_cat)
        out[f"{name}_declist_n"] = np.array(ids_n, np.int64)
        out[f"{name}_declist_dec"] = np.frombuffer(b"".join(dec), np.uint8)
        out[f"{name}_declist_dec_n"] = np.array(dn, np.int64)
    # accept / reject decisions
    good = tok_imgs["seeded"]
    small_t, small_m = [b"a", b"b", b"ab"], [(0, 1), (1, 0)]
    cases = {
        "good": good,
        "roundtrip": tok_imgs["roundtrip"],
        "bad_magic": b"XAEDNTOK" + good[8:],
        "version_1": abt(small_t, small_m, version=1),
        "version_3": abt(small_t, small_m, version=3),
        "sizes_differ": abt(small_t, small_m, declared=7),
        "file_truncated": good[:-1],
        "file_extra_byte": good + b"\0",
        "header_only": good[:64],
        "short_header": good[:40],
        "empty_file": b"",
        "checksum_wrong": abt(small_t, small_m, checksum=12345),
        "payload_flip": good[:100] + bytes([good[100] ^ 1]) + good[101:],
        "vocab_count_differs": abt(small_t, small_m, counts=(2, 2, 2)),
        "maxbytes_differs": abt(small_t, small_m, counts=(3, 9, 2)),
        "merge_count_differs": abt(small_t, small_m, counts=(3, 2, 5)),
        "block_larger_than_payload": abt(small_t, small_m, block=1 << 20),
        "block_truncated": abt(small_t, small_m, block=40),
        "offsets_truncated": abt([b"a"] * 3, [], block=6 + 8),
        "trailing_bytes": abt(small_t, small_m, extra=b"\x01\x02\x03\x04\x05"),
        "no_merges": abt(small_t, []),
        "no_tokens_no_merges": abt([], []),
        "startup_failure_fixture": b"BADMAGIC" + b"\0" * 56 + b"\0" * 16,
    }
    # merges truncated: header and payload agree on 3 rules, 2 present
    t3 = abt(small_t, small_m + [(2, 2)])
    cut = bytearray(t3[:-4])
    struct.pack_into("<Q", cut, 12, len(cut) - 64)
    struct.pack_into("<I", cut, 36, len(cut) - 64)
    struct.pack_into("<I", cut, 20, fnv1a32(bytes(cut[64:])))
    cases["merges_truncated"] = bytes(cut)
    names, oks, infos = [], [], []
    for name, img in cases.items():
        path = os.path.join(tmp, "case.abt")
        with open(path, "wb") as f:
            f.write(img)
        ok, info, _, _ = ref_run(lib, path, None, 0)
        names.append(name)
        oks.append(ok)
        infos.append(info)
        out[f"case_{name}"] = np.frombuffer(img, np.uint8)
    out["case_names"] = np.array(names)
    out["case_ok"] = np.array(oks, np.int32)
    out["case_info"] = np.stack(infos)
    path = os.path.join(HERE, "tokenizer_golden.npz")
    np.savez_compressed(path, **out)
    print(path, os.path.getsize(path), "bytes;", int(sum(oks)), "of", len(oks), "images accepted")


if __name__ == "__main__":
    sys.exit(main())
