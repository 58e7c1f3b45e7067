"""CPU restatement of the reference's .abt tokenizer: TEST INFRASTRUCTURE
ONLY (the checker for project-aaedn_b200/host/tokenizer.cpp; nothing in the
product imports it).

Follows src/tokenizer.cpp of the reference project:
  load    src/tokenizer.cpp:32-158 (header fields, checks in order, payload)
  encode  src/tokenizer.cpp:169-239 (byte tokens, linear rule scan, a
          std::priority_queue of (rule, pos, a, b) ordered by rule alone)
  decode  src/tokenizer.cpp:241-257
Pinned against the reference itself (oracle/_ref, compiled from those
sources) through tests/golden/tokenizer_golden.npz.

The queue's tie order matters (two entries with the same rule can overlap),
so the heap here is the binary heap of the C++ standard library that the
reference is built with (libstdc++): push = append, then move the new item
up while its parent compares less; pop = move the last item out, move the
top to the end, then walk the hole from the root down, always to the child
that does not compare less than its sibling (the right one when they are
equal), refill the hole with the last child of an even-length heap, and
finally move the saved item up from the hole as in push. "Compares less"
is the reference's MergeItem order: a < b when a.rule > b.rule.
"""
import struct

TOKEN_BOS, TOKEN_EOS, TOKEN_PAD = 32765, 32766, 32767


def fnv1a32(data, h=0x811C9DC5):
    for b in data:
        h ^= b
        h = (h * 0x01000193) & 0xFFFFFFFF
    return h


def load(img):
    """dict of the tables, or None where the reference returns an empty
    Tokenizer (src/tokenizer.cpp:32-158)."""
    img = bytes(img)
    if len(img) < 64:
        return None
    magic = img[:8]
    version, payload_size, checksum, vocab, max_bytes, merges, declared = struct.unpack_from("<IQI4I", img, 8)
    if magic != b"AAEDNTOK" or version != 2 or payload_size != declared:
        return None
    if len(img) - 64 != payload_size:
        return None
    payload = img[64:]
    if payload_size == 0:
        return None
    if fnv1a32(payload) != checksum:
        return None
    if len(payload) < 16:
        return None
    pv, pm, pc, block = struct.unpack_from("<4I", payload, 0)
    if pv != vocab or pm != max_bytes or pc != merges or block > payload_size:
        return None
    p = 16
    if len(payload) - p < block:
        return None
    strings = payload[p:p + block]
    p += block
    if len(payload) - p < 4 * vocab:
        return None
    offsets = list(struct.unpack_from(f"<{vocab}I", payload, p))
    p += 4 * vocab
    first, second = [], []
    for _ in range(merges):
        if len(payload) - p < 4:
            return None
        a, b = struct.unpack_from("<HH", payload, p)
        first.append(a)
        second.append(b)
        p += 4
    return dict(strings=strings, offsets=offsets, first=first, second=second, vocab_size=vocab,
                merge_count=merges, max_token_bytes=max_bytes, format_version=version, payload_checksum=checksum)


class _Heap:
    """The standard library's binary heap over (rule, pos, a, b) tuples, top =
    the item every other item compares less than or equal to."""

    def __init__(self):
        self.c = []

    @staticmethod
    def _less(x, y):  # MergeItem::operator< (src/tokenizer.cpp:165)
        return x[0] > y[0]

    def _up(self, hole, top, value):
        c = self.c
        parent = (hole - 1) // 2
        while hole > top and self._less(c[parent], value):
            c[hole] = c[parent]
            hole = parent
            parent = (hole - 1) // 2
        c[hole] = value

    def push(self, item):
        self.c.append(item)
        self._up(len(self.c) - 1, 0, item)

    def pop(self):
        c = self.c
        top = c[0]
        n = len(c)
        if n > 1:
            value = c[n - 1]
            c[n - 1] = c[0]
            length = n - 1
            hole, child = 0, 0
            while child < (length - 1) // 2:
                child = 2 * (child + 1)
                if self._less(c[child], c[child - 1]):
                    child -= 1
                c[hole] = c[child]
                hole = child
            if (length & 1) == 0 and child == (length - 2) // 2:
                child = 2 * (child + 1)
                c[hole] = c[child - 1]
                hole = child - 1
            self._up(hole, 0, value)
        c.pop()
        return top

    def __len__(self):
        return len(self.c)


def _first_rule(tok, x, y):
    for m in range(tok["merge_count"]):
        if tok["first"][m] == x and tok["second"][m] == y:
            return m
    return None


def encode(tok, text, add_bos):
    """src/tokenizer.cpp:169-239 (text: bytes, read up to the first NUL)."""
    text = bytes(text)
    if b"\0" in text:
        text = text[:text.index(b"\0")]
    tokens = list(text)
    q = _Heap()
    for i in range(len(tokens) - 1):
        m = _first_rule(tok, tokens[i], tokens[i + 1])
        if m is not None:
            q.push((m, i, tok["first"][m], tok["second"][m]))
    while len(q):
        rule, pos, a, b = q.pop()
        if pos + 1 >= len(tokens):
            continue
        if tokens[pos] != a or tokens[pos + 1] != b:
            continue
        tokens[pos] = tok["vocab_size"] + rule
        del tokens[pos + 1]
        if pos > 0:
            m = _first_rule(tok, tokens[pos - 1], tokens[pos])
            if m is not None:
                q.push((m, pos - 1, tok["first"][m], tok["second"][m]))
        if pos + 1 < len(tokens):
            m = _first_rule(tok, tokens[pos], tokens[pos + 1])
            if m is not None:
                q.push((m, pos, tok["first"][m], tok["second"][m]))
    if add_bos:
        tokens.insert(0, TOKEN_BOS)
    return tokens


def decode(tok, ids):
    """src/tokenizer.cpp:241-257, for offsets inside the string block."""
    out = bytearray()
    for i in ids:
        if i in (TOKEN_EOS, TOKEN_PAD) or i >= tok["vocab_size"]:
            continue
        s = tok["strings"]
        o = tok["offsets"][i]
        e = s.find(b"\0", o)
        out += s[o:e if e >= 0 else len(s)]
    return bytes(out)
