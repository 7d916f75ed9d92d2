"""Tokenizers and chat templates.

Reference: the BPE tokenizer of the runtime (aether_bpe_* in
runtime/src/lib.rs:5042-5250, 9534-9576; GGUF/tokenizer.json loading and the
GPT-2 byte map in runtime/src/serving.rs:3614-4170) and its chat templates
(aether_template_*, lib.rs:5304-5366). Provided here:
  * ``ByteTokenizer``  -- one token per byte plus specials (used with
    random-init models and the byte-level nano model);
  * ``BPETokenizer``   -- byte-level BPE from a Hugging Face ``tokenizer.json``
    (GPT-2 / Qwen2 family): byte-to-unicode map, merge ranks, added tokens;
  * ``SPMTokenizer``   -- SentencePiece vocabularies (GGUF
    ``tokenizer.ggml.model == "llama"``: Llama / Mistral SPM, Gemma): pieces
    with scores, spaces as U+2581, symbol-pair merges by score, byte fallback
    (reference: ``SpmModel``, runtime/src/serving.rs:2615-2700);
  * ``chat_template``  -- ChatML (Qwen2), Llama-3 and a plain fallback.
"""
from __future__ import annotations

import json
from functools import lru_cache

import regex as re

# Qwen2 / GPT-4-style pre-tokenisation pattern
_PRETOK = re.compile(
    r"""(?i:'s|'t|'re|'ve|'m|'ll|'d)|[^\r\n\p{L}\p{N}]?\p{L}+|\p{N}| ?[^\s\p{L}\p{N}]+[\r\n]*|\s*[\r\n]+|\s+(?!\S)|\s+"""
)


@lru_cache(maxsize=1)
def bytes_to_unicode() -> dict:
    """The GPT-2 reversible byte -> printable-unicode map."""
    bs = list(range(ord("!"), ord("~") + 1)) + list(range(ord("¡"), ord("¬") + 1)) + list(range(ord("®"), ord("ÿ") + 1))
    cs = bs[:]
    n = 0
    for b in range(256):
        if b not in bs:
            bs.append(b)
            cs.append(256 + n)
            n += 1
    return dict(zip(bs, [chr(c) for c in cs]))


class ByteTokenizer:
    """Bytes are tokens 0..255; specials follow."""

    def __init__(self, specials=("<|endoftext|>", "<|im_start|>", "<|im_end|>")):
        self.special = {s: 256 + i for i, s in enumerate(specials)}
        self.inv_special = {v: k for k, v in self.special.items()}
        self.vocab_size = 256 + len(specials)
        self.eos_id = self.special.get("<|endoftext|>")

    def encode(self, text: str, allow_special: bool = True) -> list:
        out = []
        if allow_special and self.special:
            pat = re.compile("(" + "|".join(re.escape(s) for s in self.special) + ")")
            parts = pat.split(text)
        else:
            parts = [text]
        for part in parts:
            if part in self.special and allow_special:
                out.append(self.special[part])
            elif part:
                out.extend(part.encode("utf-8"))
        return out

    def decode(self, ids) -> str:
        buf = bytearray()
        out = []
        for i in ids:
            i = int(i)
            if i < 256:
                buf.append(i)
            else:
                out.append(buf.decode("utf-8", errors="replace"))
                buf = bytearray()
                out.append(self.inv_special.get(i, ""))
        out.append(buf.decode("utf-8", errors="replace"))
        return "".join(out)


class BPETokenizer:
    def __init__(self, vocab: dict, merges: list, added_tokens: dict | None = None):
        self.vocab = vocab
        self.inv = {v: k for k, v in vocab.items()}
        self.ranks = {tuple(m.split(" ", 1)) if isinstance(m, str) else tuple(m): i for i, m in enumerate(merges)}
        self.special = dict(added_tokens or {})
        for k, v in self.special.items():
            self.inv[v] = k
        self.vocab_size = max(self.inv) + 1 if self.inv else 0
        self.byte_enc = bytes_to_unicode()
        self.byte_dec = {v: k for k, v in self.byte_enc.items()}
        self.eos_id = self.special.get("<|endoftext|>", self.special.get("<|im_end|>"))
        self._cache: dict = {}

    @staticmethod
    def from_file(path: str) -> "BPETokenizer":
        with open(path, encoding="utf-8") as f:
            tj = json.load(f)
        model = tj["model"]
        added = {t["content"]: t["id"] for t in tj.get("added_tokens", [])}
        return BPETokenizer(model["vocab"], model.get("merges", []), added)

    def _bpe(self, word: str) -> list:
        if word in self._cache:
            return self._cache[word]
        parts = list(word)
        while len(parts) > 1:
            best, best_i = None, -1
            for i in range(len(parts) - 1):
                r = self.ranks.get((parts[i], parts[i + 1]))
                if r is not None and (best is None or r < best):
                    best, best_i = r, i
            if best is None:
                break
            parts = parts[:best_i] + [parts[best_i] + parts[best_i + 1]] + parts[best_i + 2 :]
        self._cache[word] = parts
        return parts

    def encode(self, text: str, allow_special: bool = True) -> list:
        out = []
        if allow_special and self.special:
            pat = re.compile("(" + "|".join(re.escape(s) for s in sorted(self.special, key=len, reverse=True)) + ")")
            chunks = pat.split(text)
        else:
            chunks = [text]
        for chunk in chunks:
            if not chunk:
                continue
            if allow_special and chunk in self.special:
                out.append(self.special[chunk])
                continue
            for piece in _PRETOK.findall(chunk):
                mapped = "".join(self.byte_enc[b] for b in piece.encode("utf-8"))
                for tok in self._bpe(mapped):
                    tid = self.vocab.get(tok)
                    if tid is None:  # unknown merge result: fall back to single symbols
                        out.extend(self.vocab[c] for c in tok if c in self.vocab)
                    else:
                        out.append(tid)
        return out

    def decode(self, ids) -> str:
        text = []
        buf = bytearray()
        for i in ids:
            tok = self.inv.get(int(i), "")
            if tok in self.special:
                text.append(buf.decode("utf-8", errors="replace"))
                buf = bytearray()
                text.append(tok)
                continue
            for ch in tok:
                b = self.byte_dec.get(ch)
                if b is not None:
                    buf.append(b)
        text.append(buf.decode("utf-8", errors="replace"))
        return "".join(text)


_SPACE = "\u2581"


class SPMTokenizer:
    """SentencePiece tokenizer of the score-merge kind llama.cpp uses for
    ``llama``-model GGUF vocabularies.

    Encoding: spaces become U+2581 (optionally one is prefixed), the text is
    split into UTF-8 characters, and the adjacent pair whose concatenation is
    the highest-scoring vocabulary piece is merged repeatedly (ties: the
    leftmost pair) until no adjacent pair forms a piece; a symbol that is not
    a piece falls back to its ``<0xNN>`` byte tokens. This is SentencePiece's
    BPE-model encoding, which the Llama / Mistral / Gemma vocabularies use.
    Control and unused entries (token types 3 and 5) take no part in merging;
    user-defined / control strings (types 3, 4) are matched whole first.
    """

    NORMAL, UNKNOWN, CONTROL, USER, UNUSED, BYTE = 1, 2, 3, 4, 5, 6

    def __init__(self, pieces: list, scores: list, types: list | None = None, bos_id: int | None = None,
                 eos_id: int | None = None, add_bos: bool = False, add_space_prefix: bool = False,
                 unk_id: int | None = None):
        types = list(types) if types is not None else [self.NORMAL] * len(pieces)
        self.pieces = list(pieces)
        self.vocab_size = len(pieces)
        self.piece_id: dict = {}
        self.score: dict = {}
        self.byte_id = [-1] * 256
        self.special: dict = {}
        for i, (p, sc, ty) in enumerate(zip(self.pieces, scores, types)):
            if len(p) == 6 and p.startswith("<0x") and p.endswith(">"):
                try:
                    self.byte_id[int(p[3:5], 16)] = i
                    continue
                except ValueError:
                    pass
            if ty in (self.CONTROL, self.USER):
                if p:
                    self.special.setdefault(p, i)
                continue
            if ty == self.UNUSED or not p:
                continue
            if p not in self.piece_id:  # the lowest id wins for a repeated surface
                self.piece_id[p] = i
                self.score[p] = float(sc)
        self.bos_id, self.eos_id, self.unk_id = bos_id, eos_id, unk_id
        self.add_bos, self.add_space_prefix = add_bos, add_space_prefix
        self._special_re = (re.compile("(" + "|".join(re.escape(t) for t in sorted(self.special, key=len,
                                                                                    reverse=True)) + ")")
                            if self.special else None)

    @staticmethod
    def from_sentencepiece(model_file: str, **kw) -> "SPMTokenizer":
        """From a SentencePiece ``.model`` file (needs the ``sentencepiece`` package)."""
        import sentencepiece as spm

        sp = spm.SentencePieceProcessor(model_file=model_file)
        n = sp.get_piece_size()
        types = []
        for i in range(n):
            types.append(SPMTokenizer.CONTROL if sp.is_control(i) else SPMTokenizer.UNKNOWN if sp.is_unknown(i)
                         else SPMTokenizer.UNUSED if sp.is_unused(i) else SPMTokenizer.BYTE if sp.is_byte(i)
                         else SPMTokenizer.NORMAL)
        return SPMTokenizer([sp.id_to_piece(i) for i in range(n)], [sp.get_score(i) for i in range(n)], types,
                            bos_id=sp.bos_id() if sp.bos_id() >= 0 else None,
                            eos_id=sp.eos_id() if sp.eos_id() >= 0 else None,
                            unk_id=sp.unk_id() if sp.unk_id() >= 0 else None, **kw)

    def _encode_fragment(self, text: str) -> list:
        import heapq

        if not text:
            return []
        text = text.replace(" ", _SPACE)
        sym = list(text)  # one symbol per character; "" marks a symbol merged away
        n = len(sym)
        prev = list(range(-1, n - 1))
        nxt = list(range(1, n + 1))
        nxt[-1] = -1
        heap = []

        def push(i, j):
            if i < 0 or j < 0:
                return
            cand = sym[i] + sym[j]
            sc = self.score.get(cand)
            if sc is not None:
                heapq.heappush(heap, (-sc, i, j, cand))

        for i in range(n - 1):
            push(i, i + 1)
        while heap:
            _, i, j, cand = heapq.heappop(heap)
            if not sym[i] or not sym[j] or nxt[i] != j or sym[i] + sym[j] != cand:
                continue  # stale: one side was merged since this pair was queued
            sym[i] = cand
            sym[j] = ""
            nxt[i] = nxt[j]
            if nxt[j] >= 0:
                prev[nxt[j]] = i
            push(prev[i], i)
            push(i, nxt[i])
        out = []
        i = 0
        while i >= 0 and i < n:
            s = sym[i]
            tid = self.piece_id.get(s)
            if tid is not None:
                out.append(tid)
            else:  # byte fallback
                for b in s.encode("utf-8"):
                    bid = self.byte_id[b]
                    out.append(bid if bid >= 0 else (self.unk_id if self.unk_id is not None else 0))
            i = nxt[i]
        return out

    def encode(self, text: str, allow_special: bool = True, add_bos: bool | None = None) -> list:
        out = [self.bos_id] if (self.add_bos if add_bos is None else add_bos) and self.bos_id is not None else []
        parts = self._special_re.split(text) if (allow_special and self._special_re) else [text]
        after_special = True  # a text fragment at the start or after a special token gets the space prefix
        for part in parts:
            if not part:
                continue
            if allow_special and part in self.special:
                out.append(self.special[part])
                after_special = True
                continue
            if after_special and self.add_space_prefix:
                part = " " + part
            after_special = False
            out.extend(self._encode_fragment(part))
        return out

    def decode(self, ids) -> str:
        buf = bytearray()
        for i in ids:
            i = int(i)
            if not 0 <= i < self.vocab_size:
                continue
            p = self.pieces[i]
            if len(p) == 6 and p.startswith("<0x") and p.endswith(">") and self.byte_id[int(p[3:5], 16)] == i:
                buf.append(int(p[3:5], 16))
            elif i in (self.bos_id, self.eos_id) or (p in self.special and self.special[p] == i
                                                      and p.startswith("<") and p.endswith(">")):
                continue  # control tokens render as nothing
            else:
                buf.extend(p.replace(_SPACE, " ").encode("utf-8"))
        text = buf.decode("utf-8", errors="replace")
        if self.add_space_prefix and text.startswith(" "):
            text = text[1:]  # the space the encoder prefixed
        return text


def chat_template(messages: list, style: str = "chatml", add_generation_prompt: bool = True) -> str:
    """Renders OpenAI-style messages ({role, content}) into a prompt string."""
    out = []
    if style == "chatml":
        for m in messages:
            out.append(f"<|im_start|>{m['role']}\n{m.get('content', '')}<|im_end|>\n")
        if add_generation_prompt:
            out.append("<|im_start|>assistant\n")
    elif style == "llama3":
        out.append("<|begin_of_text|>")
        for m in messages:
            out.append(f"<|start_header_id|>{m['role']}<|end_header_id|>\n\n{m.get('content', '')}<|eot_id|>")
        if add_generation_prompt:
            out.append("<|start_header_id|>assistant<|end_header_id|>\n\n")
    else:
        for m in messages:
            out.append(f"{m['role']}: {m.get('content', '')}\n")
        if add_generation_prompt:
            out.append("assistant: ")
    return "".join(out)
