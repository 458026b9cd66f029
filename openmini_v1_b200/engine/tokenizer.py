"""Tokenizer.

Two forms, chosen by what the checkpoint provides:

* GGUF vocabulary (``tokenizer.ggml.tokens`` / ``scores`` / ``token_type`` /
  ``merges``): SentencePiece-style pieces with ``▁`` as the space marker and
  ``<0xNN>`` byte-fallback pieces. Encoding is BPE over merge ranks when
  ``merges`` are present, else greedy longest-match over the vocabulary
  (a trie), falling back to byte pieces for anything unknown.
* Byte-level (random-init models): id = 3 + byte, with <unk>=0, <s>=1, </s>=2.

Mirrors the capabilities of openmini-server/src/model/inference/tokenizer.rs
(load_from_gguf 436, encode 605, decode 827): special tokens, batch
encode/decode and streaming-safe incremental decode.
"""
from __future__ import annotations

import re

SPACE = "▁"


class ByteTokenizer:
    unk_id, bos_id, eos_id = 0, 1, 2

    def __init__(self, vocab_size: int = 32000):
        self.vocab_size = vocab_size

    def encode(self, text: str, add_bos: bool = True) -> list:
        ids = [3 + b for b in text.encode("utf-8")]
        return ([self.bos_id] if add_bos else []) + ids

    def decode(self, ids, skip_special: bool = True) -> str:
        out = bytearray()
        for i in ids:
            i = int(i)
            if 3 <= i < 259:
                out.append(i - 3)
            elif not skip_special:
                out += f"<{i}>".encode()
            # ids >= 259 have no byte meaning in a random-init model: render as nothing
        return out.decode("utf-8", errors="replace")

    def decode_token(self, i: int) -> bytes:
        i = int(i)
        return bytes([i - 3]) if 3 <= i < 259 else b""

    def batch_encode(self, texts, add_bos=True):
        return [self.encode(t, add_bos) for t in texts]

    def batch_decode(self, seqs):
        return [self.decode(s) for s in seqs]


class GGUFTokenizer:
    dummy_prefix = True  # encode() prepends the SentencePiece space marker

    def __init__(self, tokens, scores=None, token_types=None, merges=None, bos_id=1, eos_id=2, unk_id=0):
        self.tokens = list(tokens)
        self.vocab_size = len(self.tokens)
        self.index = {t: i for i, t in enumerate(self.tokens)}
        self.scores = scores
        self.types = token_types
        self.bos_id, self.eos_id, self.unk_id = bos_id, eos_id, unk_id
        self.byte_ids = {}
        for i, t in enumerate(self.tokens):
            m = re.fullmatch(r"<0x([0-9A-Fa-f]{2})>", t)
            if m:
                self.byte_ids[int(m.group(1), 16)] = i
        self.ranks = None
        if merges:
            self.ranks = {tuple(m.split(" ", 1)): r for r, m in enumerate(merges) if " " in m}
        self.trie = {}
        for i, t in enumerate(self.tokens):
            if self.types is not None and self.types[i] in (2, 3, 4):  # unknown / control / user-defined
                continue
            node = self.trie
            for ch in t:
                node = node.setdefault(ch, {})
            node[None] = i

    @staticmethod
    def from_gguf(reader) -> "GGUFTokenizer":
        md = reader.metadata
        return GGUFTokenizer(md["tokenizer.ggml.tokens"], md.get("tokenizer.ggml.scores"),
                             md.get("tokenizer.ggml.token_type"), md.get("tokenizer.ggml.merges"),
                             int(md.get("tokenizer.ggml.bos_token_id", 1)), int(md.get("tokenizer.ggml.eos_token_id", 2)),
                             int(md.get("tokenizer.ggml.unknown_token_id", 0)))

    def _pieces_for(self, s: str) -> list:
        if self.ranks:
            return self._bpe(s)
        return self._greedy(s)

    def _greedy(self, s: str) -> list:
        out, i = [], 0
        while i < len(s):
            node, j, best, best_j = self.trie, i, None, i
            while j < len(s) and s[j] in node:
                node = node[s[j]]
                j += 1
                if None in node:
                    best, best_j = node[None], j
            if best is None:
                out += self._bytes(s[i])
                i += 1
            else:
                out.append(best)
                i = best_j
        return out

    def _bpe(self, s: str) -> list:
        parts = list(s)
        while len(parts) > 1:
            best, bi = None, -1
            for k in range(len(parts) - 1):
                r = self.ranks.get((parts[k], parts[k + 1]))
                if r is not None and (best is None or r < best):
                    best, bi = r, k
            if best is None:
                break
            parts[bi:bi + 2] = [parts[bi] + parts[bi + 1]]
        out = []
        for p in parts:
            if p in self.index:
                out.append(self.index[p])
            else:
                for ch in p:
                    out += self._bytes(ch)
        return out

    def _bytes(self, ch: str) -> list:
        if ch in self.index:
            return [self.index[ch]]
        ids = [self.byte_ids.get(b) for b in ch.encode("utf-8")]
        return [i if i is not None else self.unk_id for i in ids]

    def encode(self, text: str, add_bos: bool = True) -> list:
        s = SPACE + text.replace(" ", SPACE)
        return ([self.bos_id] if add_bos else []) + self._pieces_for(s)

    def decode_token(self, i: int) -> bytes:
        i = int(i)
        if i < 0 or i >= self.vocab_size:
            return b""
        t = self.tokens[i]
        m = re.fullmatch(r"<0x([0-9A-Fa-f]{2})>", t)
        if m:
            return bytes([int(m.group(1), 16)])
        if self.types is not None and self.types[i] == 3:
            return b""
        return t.replace(SPACE, " ").encode("utf-8")

    def decode(self, ids, skip_special: bool = True) -> str:
        b = b"".join(self.decode_token(i) for i in ids if not (skip_special and i in (self.bos_id, self.eos_id)))
        s = b.decode("utf-8", errors="replace")
        return s[1:] if s.startswith(" ") else s

    def batch_encode(self, texts, add_bos=True):
        return [self.encode(t, add_bos) for t in texts]

    def batch_decode(self, seqs):
        return [self.decode(s) for s in seqs]


class IncrementalDecoder:
    """Streams text from token ids without splitting multi-byte UTF-8 characters. For a
    tokenizer that prepends a dummy space (``dummy_prefix``), the first character of the
    stream is dropped when it is that space, as ``decode`` does for the whole text."""

    def __init__(self, tok):
        self.tok = tok
        self.buf = b""
        self._strip = bool(getattr(tok, "dummy_prefix", False))

    def _emit(self, s: str) -> str:
        if self._strip and s:
            self._strip = False
            if s[0] == " ":
                return s[1:]
        return s

    def push(self, token_id: int) -> str:
        self.buf += self.tok.decode_token(token_id)
        try:
            s = self.buf.decode("utf-8")
            self.buf = b""
            return self._emit(s)
        except UnicodeDecodeError as e:
            if e.start > 0:
                s = self.buf[:e.start].decode("utf-8")
                self.buf = self.buf[e.start:]
                return self._emit(s)
            if len(self.buf) > 4:  # not a truncated character: emit replacement
                s = self.buf.decode("utf-8", errors="replace")
                self.buf = b""
                return self._emit(s)
            return ""
