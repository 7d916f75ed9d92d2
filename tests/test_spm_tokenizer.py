"""SentencePiece tokenizer against the sentencepiece package: a BPE-type
model with byte fallback is trained here on a small seeded corpus (the kind of
model Llama / Mistral / Gemma GGUF vocabularies come from), and the encodings
of this package's SPMTokenizer must equal sentencepiece's, id for id, with
and without the dummy space prefix; decoding round-trips, including bytes
that fall back to <0xNN> tokens. A GGUF file written with the vocabulary
loads back as the same tokenizer."""
import os
import random

import pytest

spm = pytest.importorskip("sentencepiece")

from aether_b200.serving.tokenizer import SPMTokenizer  # noqa: E402

WORDS = ("the quick brown fox jumps over lazy dog tensor parallel decode prefill attention kernel "
         "blackwell memory bandwidth token model serving server request user assistant hello world").split()
TEXTS = ["hello world", " the quick brown fox", "tensor  parallel   decode", "Hello World!", "user: hi",
         "naïve café ünïcode 東京", "xyzzy qwerty", "dog\nnew line\ttab", "", " ", "a"]


def _train(tmp, prefix):
    rnd = random.Random(0)
    corpus = os.path.join(tmp, "corpus.txt")
    with open(corpus, "w") as f:
        for _ in range(3000):
            f.write(" ".join(rnd.choice(WORDS) for _ in range(rnd.randint(3, 12))) + "\n")
    base = os.path.join(tmp, f"m{int(prefix)}")
    spm.SentencePieceTrainer.train(input=corpus, model_prefix=base, vocab_size=300, model_type="bpe",
                                   byte_fallback=True, normalization_rule_name="identity",
                                   add_dummy_prefix=prefix, remove_extra_whitespaces=False, character_coverage=1.0, bos_id=1, eos_id=2, unk_id=0,
                                   minloglevel=2)
    return base + ".model"


@pytest.mark.parametrize("prefix", [False, True])
def test_spm_matches_sentencepiece(tmp_path, prefix):
    model = _train(str(tmp_path), prefix)
    sp = spm.SentencePieceProcessor(model_file=model)
    tok = SPMTokenizer.from_sentencepiece(model, add_space_prefix=prefix)
    for t in TEXTS:
        want = sp.encode(t)
        got = tok.encode(t, add_bos=False)
        assert got == want, (t, got, want, [sp.id_to_piece(i) for i in want])
        assert tok.decode(got) == sp.decode(want), t
    assert tok.encode("hello", add_bos=True)[0] == sp.bos_id()


def test_spm_from_gguf_metadata(tmp_path):
    from aether_b200.formats import gguf as G

    model = _train(str(tmp_path), True)
    sp = spm.SentencePieceProcessor(model_file=model)
    ref = SPMTokenizer.from_sentencepiece(model, add_space_prefix=True)
    n = sp.get_piece_size()
    types = [3 if sp.is_control(i) else 2 if sp.is_unknown(i) else 6 if sp.is_byte(i) else 1 for i in range(n)]
    meta = {"general.architecture": "llama", "tokenizer.ggml.model": "llama",
            "tokenizer.ggml.tokens": [sp.id_to_piece(i) for i in range(n)],
            "tokenizer.ggml.scores": [float(sp.get_score(i)) for i in range(n)],
            "tokenizer.ggml.token_type": types, "tokenizer.ggml.bos_token_id": 1, "tokenizer.ggml.eos_token_id": 2,
            "tokenizer.ggml.unknown_token_id": 0, "tokenizer.ggml.add_bos_token": True,
            "tokenizer.ggml.add_space_prefix": True}
    path = os.path.join(str(tmp_path), "tok.gguf")
    G.write_gguf(path, meta, {})
    tok = G.tokenizer_from_gguf(G.GGUFFile(path))
    assert isinstance(tok, SPMTokenizer)
    for t in TEXTS:
        assert tok.encode(t) == [1] + ref.encode(t, add_bos=False), t
        assert tok.encode(t) == [1] + sp.encode(t), t
