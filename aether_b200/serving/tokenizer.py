"""Tokenizers and chat templates.

Reference: the BPE tokenizer of the runtime (aether_bpe_* in
runtime/src/lib.rs:5042-5250, 9534-9576; GGUF/tokenizer.json loading and the
GPT-2 byte map in runtime/src/serving.rs:3614-4170) and its chat templates
(aether_template_*, lib.rs:5304-5366). Provided here:
  * ``ByteTokenizer``  -- one token per byte plus specials (used with
    random-init models and the byte-level nano model);
  * ``BPETokenizer``   -- byte-level BPE from a Hugging Face ``tokenizer.json``
    (GPT-2 / Qwen2 family): byte-to-unicode map, merge ranks, added tokens;
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
