"""Generates tests/golden/tokenizer_ref.json: token ids from the reference's own
BGETokenizer (src/tokenizer.cpp compiled unmodified into oracle/_ref/libfe_ref_tok.so by
oracle/Makefile) with the [CLS] / [SEP] framing of SentenceTransformerImpl::tokenize.

    python __graft_entry__.py && python tests/golden/gen_golden_tokenizer.py

The vocabulary is tests/model_dir.py's synthetic one (plus one repeated line); the texts
are tests/test_tokenizer.py's fixed cases and its seeded random byte strings.
"""
from __future__ import annotations

import json
import os
import sys
import tempfile

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle.oracle import RefTokenizer  # noqa: E402
from tests import test_tokenizer as T  # noqa: E402


def main() -> None:
    if not RefTokenizer.available():
        sys.exit("oracle/_ref/libfe_ref_tok.so is not built (needs the reference sources)")
    with tempfile.TemporaryDirectory() as d:
        path = T.write_vocab(d)
        ref = RefTokenizer(path)
        cases = [{"text": t.hex(), "ids": ref.encode(t)} for t in T.golden_texts()]
        ref.close()
    with open(os.path.join(HERE, "tokenizer_ref.json"), "w") as f:
        json.dump({"vocab_size": T.VOCAB_SIZE, "cases": cases}, f, separators=(",", ":"))
    print(f"{len(cases)} cases")


if __name__ == "__main__":
    main()
