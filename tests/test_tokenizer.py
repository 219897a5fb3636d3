"""The drop-in BGE WordPiece tokenizer (fe_wordpiece_*, the tokenizer of the C++
SentenceTransformer) against the reference's own BGETokenizer (src/tokenizer.cpp,
compiled unmodified into oracle/_ref/libfe_ref_tok.so), token for token, with the
[CLS] / [SEP] framing of SentenceTransformerImpl::tokenize
(src/sentence_transformers_impl.cpp:11-27).  Host only: no GPU.

Two checks: the committed ids the reference produced (tests/golden/tokenizer_ref.json,
made by tests/golden/gen_golden_tokenizer.py), which hold wherever the reference
sources are absent, and, where oracle/_ref/libfe_ref_tok.so was built, the live
reference on a larger seeded set of random byte strings."""
import ctypes as C
import json
import os

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
VOCAB_SIZE = 21128

FIXED = [
    "Hello world!", "the cat sat on the mat.", "Embeddings, fast: B200 GPU model", "一丁七万丈三上下",
    "unknownwordzzz and   spaces\tand-tabs", "a", "embedding embeddings embedder", "x" * 40,
    "mixed 中文 text, with ‘quotes’ and émojis 🙂", "", "   ", "\t\n\v\f\r", "UPPER lower MiXeD 123 4x4",
    "[UNK] [CLS] [SEP] ##s ##ding", "catsat matcat thecat", "embedd embeddingsembedding", "!!!???...---",
    "ab\x00cd", "tab\tsep\rcr\nnl",
]
RAW = [
    b"\x80", b"\xbf\xbf", b"\xff", b"\xfe abc", b"\xc0", b"\xc3", b"abc\xe4\xb8", b"\xe4\xb8\x80\xe4", b"\xf0\x9f",
    b"\xf8\x88\x80\x80\x80", b"cat\x80sat", b"sat\xe4\xb8\x80mat", b"\xc3\xa9t\xc3\xa9", b"\xe4a\x80b",
    b"hello\xffworld", b"\xe4\xb8\x80" * 20, b"GPU\xf0\x9f\x99\x82gpu", b"x\xc3",
]
ALPHABET = (list(b"abcdefghijklmnopqrstuvwxyzABCXYZ0123456789 \t\n.,!?-'#[]") +
            [0x80, 0xA9, 0xBF, 0xC3, 0xE4, 0xB8, 0xF0, 0x9F, 0xFF, 0x00])


def write_vocab(d):
    from tests.model_dir import synthetic_vocab
    v = synthetic_vocab(VOCAB_SIZE)
    v[2000] = "cat"  # a repeated line: the later id wins, as a map assignment does
    path = os.path.join(d, "vocab.txt")
    with open(path, "w", encoding="utf-8") as f:
        f.write("\n".join(v) + "\n")
    return path


def random_texts(n, seed):
    rng = np.random.default_rng(seed)
    out = []
    for _ in range(n):
        L = int(rng.integers(0, 48))
        out.append(bytes(int(ALPHABET[i]) for i in rng.integers(0, len(ALPHABET), size=L)))
    return out


def golden_texts():
    return [t.encode("utf-8") for t in FIXED] + RAW + random_texts(300, seed=7)


class Product:
    """fe_wordpiece_* of libfastembed_b200.so (host only)."""

    def __init__(self, vocab_path):
        from fastembed_b200 import capi
        self.L = capi.lib()
        self.h = C.c_void_p()
        capi.check(self.L.fe_wordpiece_create(vocab_path.encode(), C.byref(self.h)), "fe_wordpiece_create")

    def encode(self, text: bytes):
        n = C.c_size_t(0)
        assert self.L.fe_wordpiece_encode(self.h, text, len(text), None, 0, C.byref(n)) == 0
        buf = (C.c_int32 * n.value)()
        m = C.c_size_t(0)
        assert self.L.fe_wordpiece_encode(self.h, text, len(text), buf, n.value, C.byref(m)) == 0
        assert m.value == n.value
        return list(buf)

    def close(self):
        self.L.fe_wordpiece_destroy(self.h)


@pytest.fixture(scope="module")
def vocab_path(tmp_path_factory, fe_lib):
    return write_vocab(str(tmp_path_factory.mktemp("vocab")))


def test_matches_reference_golden_ids(vocab_path):
    with open(os.path.join(HERE, "golden", "tokenizer_ref.json")) as f:
        gold = json.load(f)
    assert gold["vocab_size"] == VOCAB_SIZE
    texts = golden_texts()
    assert [c["text"] for c in gold["cases"]] == [t.hex() for t in texts], "text set changed"
    p = Product(vocab_path)
    for t, c in zip(texts, gold["cases"]):
        assert p.encode(t) == c["ids"], t
    p.close()


def test_matches_live_reference(vocab_path):
    from oracle.oracle import RefTokenizer
    if not RefTokenizer.available():
        pytest.skip("oracle/_ref/libfe_ref_tok.so not built (reference sources absent); the golden ids still pin it")
    ref = RefTokenizer(vocab_path)
    p = Product(vocab_path)
    for t in golden_texts() + random_texts(3000, seed=8):
        assert p.encode(t) == ref.encode(t), t
    ref.close()
    p.close()


def test_errors(tmp_path, fe_lib):
    h = C.c_void_p()
    assert fe_lib.fe_wordpiece_create(str(tmp_path / "missing.txt").encode(), C.byref(h)) == 6  # FE_ERR_IO
    bad = tmp_path / "no_unk.txt"
    bad.write_text("[PAD]\nhello\n")
    assert fe_lib.fe_wordpiece_create(str(bad).encode(), C.byref(h)) == 6
    assert b"[UNK]" in fe_lib.fe_last_error_message()
    assert fe_lib.fe_wordpiece_create(None, C.byref(h)) == 1
