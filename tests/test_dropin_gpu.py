"""The drop-in C++ boundary on a B200.

* The reference's own GTest files (tests/matrix_ops_test.cpp, tests/attention_ops_test.cpp),
  compiled unmodified against this repository's CUDAMatrixOps / CUDAAttentionOps (by
  oracle/Makefile, into oracle/_ref/), must pass: GEMM, activations and LayerNorm within
  1e-5 and attention within 1e-3 of the reference CPU ops.
* SentenceTransformer(model_dir) built from config.json, vocab.txt and model.safetensors
  (F32 or BF16 entries) must tokenize exactly as the reference's WordPiece does and embed
  within the stated tolerance of the oracle forward; encode() of one text must equal its
  row of encode_batch() bit for bit; FE_DEVICES="0,0" (two engines, two host threads,
  cost-balanced slices) must give the same bits as one engine.
"""
import dataclasses
import os
import subprocess

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_BIN = os.path.join(ROOT, "oracle", "_ref")

TEXTS = [
    "Hello world!",
    "the cat sat on the mat.",
    "Embeddings, fast: B200 GPU model",
    "一丁七万丈三上下",
    "unknownwordzzz and   spaces\tand-tabs",
    "a",
    "embedding embeddings embedder",
    "x" * 40,
    "mixed 中文 text, with ‘quotes’ and émojis 🙂",
]


@pytest.mark.parametrize("name", ["matrix_ops_test", "attention_ops_test"])
def test_reference_gtests_pass_on_dropin(cuda_dev, name):
    exe = os.path.join(REF_BIN, name)
    if not os.path.exists(exe):
        pytest.skip(f"{exe} was not built (needs the reference sources at build time)")
    r = subprocess.run([exe], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-2000:]
    assert ", 0 failed" in r.stdout


def _st_check():
    exe = os.path.join(ROOT, "tests", "cpp", "st_check")
    subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "tests", "cpp")], check=True)
    return exe


def _run_model(tmp_path, dtype, env_extra=None):
    from fastembed_b200 import workload as W
    from tests.model_dir import bf16_round_trip, write_model_dir
    shape = dataclasses.replace(W.SHAPES["bge-small"], layers=2)
    weights = W.make_weights(shape, seed=11)
    mdir = str(tmp_path / f"model_{dtype}")
    vocab = write_model_dir(mdir, shape, weights, dtype)
    texts = tmp_path / "texts.txt"
    texts.write_text("\n".join(TEXTS) + "\n", encoding="utf-8")
    pre = str(tmp_path / f"out_{dtype}")
    env = dict(os.environ)
    env.update(env_extra or {})
    r = subprocess.run([_st_check(), mdir, str(texts), pre], capture_output=True, text=True, env=env, timeout=600)
    assert r.returncode == 0, r.stderr
    raw = np.fromfile(pre + ".ids", dtype=np.int32)
    ids, i = [], 0
    while i < raw.size:
        n = int(raw[i])
        ids.append(raw[i + 1:i + 1 + n].copy())
        i += 1 + n
    D = shape.hidden
    batch = np.fromfile(pre + ".batch", dtype=np.float32).reshape(-1, D)
    single = np.fromfile(pre + ".single", dtype=np.float32).reshape(-1, D)
    concurrent = np.fromfile(pre + ".concurrent", dtype=np.float32).reshape(-1, D)
    assert np.array_equal(concurrent, single)  # threads sharing the object: merged batches, same rows
    # the texts 40 times in one batch, tokenised on several host threads: every repetition
    # gives the same rows; against the small batch (which runs the 1-CTA GEMM and the
    # two-launch norm instead of the 2-CTA GEMM and the fused norm) within fp32 rounding
    big = np.fromfile(pre + ".big", dtype=np.float32).reshape(40, -1, D)
    assert all(np.array_equal(big[0], big[r]) for r in range(1, 40))
    assert np.abs(big[0] - batch).max() <= 1e-5
    used = weights if dtype == "F32" else {k: bf16_round_trip(v) for k, v in weights.items()}
    return shape, vocab, used, ids, batch, single


@pytest.mark.parametrize("dtype", ["F32", "BF16"])
def test_sentence_transformer_dropin(cuda_dev, oracle_lib, tmp_path, dtype):
    from oracle.wordpiece import WordPiece
    shape, vocab, weights, ids, batch, single = _run_model(tmp_path, dtype)
    wp = WordPiece(vocab)
    for text, got in zip(TEXTS, ids):
        assert got.tolist() == wp.encode(text), text
    model = oracle_lib.Model(shape, weights)
    lengths = np.array([len(x) for x in ids], np.int32)
    padded = np.zeros((len(ids), int(lengths.max())), np.int32)
    for b, x in enumerate(ids):
        padded[b, :len(x)] = x
    ref = model.forward_batch(padded, lengths)
    cos = (batch * ref).sum(1) / (np.linalg.norm(batch, axis=1) * np.linalg.norm(ref, axis=1))
    assert cos.min() >= 0.9999 and np.abs(batch - ref).max() <= 2e-3
    assert np.array_equal(single, batch)  # one text alone == its row of the batch


def test_multi_engine_slices_are_bit_identical(cuda_dev, tmp_path):
    _, _, _, _, one, _ = _run_model(tmp_path / "one", "F32")
    _, _, _, _, two, _ = _run_model(tmp_path / "two", "F32", {"FE_DEVICES": "0,0"})
    assert np.array_equal(one, two)


def test_sentence_transformer_bge_m3_ids(cuda_dev, oracle_lib, tmp_path):
    """A bge-m3 model directory (model_type "xlm-roberta", pad_token_id 1) through the C++
    SentenceTransformer: encode_ids matches the oracle's XLM-R position path, and text is
    refused (the SentencePiece tokenizer is not part of this build)."""
    from fastembed_b200 import workload as W
    from tests.model_dir import write_model_dir
    shape = dataclasses.replace(W.SHAPES["bge-small"], layers=2, max_pos=64, type_vocab=1, pad_id=1)
    weights = W.make_weights(shape, seed=31)
    mdir = str(tmp_path / "m3")
    write_model_dir(mdir, shape, weights, "F32")
    lengths = np.array([3, 9, 60, 64, 20], np.int32)
    ids, _ = W.sample_ids(shape, lengths, seed=32, pad_to=64)
    ids[1, 4] = 1
    ids[4, 2:6] = 1
    seqs = [ids[b, :lengths[b]] for b in range(len(lengths))]
    raw = np.concatenate([np.concatenate([[len(x)], x]) for x in seqs]).astype(np.int32)
    (tmp_path / "ids.bin").write_bytes(raw.tobytes())
    pre = str(tmp_path / "out")
    r = subprocess.run([_st_check(), mdir, str(tmp_path / "ids.bin"), pre, "ids"], capture_output=True, text=True,
                       timeout=600)
    assert r.returncode == 0, r.stderr
    assert "text rejected 1" in r.stdout
    got = np.fromfile(pre + ".batch", dtype=np.float32).reshape(-1, shape.hidden)
    ref = oracle_lib.Model(shape, weights).forward_batch(ids, lengths)
    cos = (got * ref).sum(1) / (np.linalg.norm(got, axis=1) * np.linalg.norm(ref, axis=1))
    assert cos.min() >= 0.9999 and np.abs(got - ref).max() <= 2e-3
