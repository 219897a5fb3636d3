"""Writes a model directory in the reference's on-disk format (config.json, vocab.txt,
model.safetensors) from seeded synthetic weights, for the drop-in SentenceTransformer
tests.  The vocabulary is made up: [PAD]=0, [UNK]=100, [CLS]=101, [SEP]=102, ASCII letters
and digits, a few "##" continuations and some CJK characters, padded to vocab_size."""
from __future__ import annotations

import json
import os
import struct

import numpy as np


def synthetic_vocab(size: int) -> list[str]:
    v = [f"[unused{i}]" for i in range(size)]
    v[0], v[100], v[101], v[102] = "[PAD]", "[UNK]", "[CLS]", "[SEP]"
    words = ["the", "cat", "sat", "on", "mat", "embed", "##ding", "##s", "fast", "b200", "gpu", "model", "##er",
             "hello", "world", ".", ",", "!", "?", "-", "'", "a", "an", "is", "of", "to", "in"]
    words += [chr(c) for c in range(ord("a"), ord("z") + 1)] + [str(d) for d in range(10)]
    words += ["##" + chr(c) for c in range(ord("a"), ord("z") + 1)]
    words += [chr(0x4E00 + i) for i in range(200)]  # CJK characters
    for i, w in enumerate(words):
        v[1000 + i] = w
    return v


def write_safetensors(path: str, tensors: dict, dtype: str = "F32") -> None:
    header, blobs, off = {}, [], 0
    for name, arr in tensors.items():
        a = np.ascontiguousarray(arr, dtype=np.float32)
        if dtype == "BF16":
            raw = (a.view(np.uint32) >> 16).astype(np.uint16).tobytes()  # truncating widen-able bf16
        else:
            raw = a.tobytes()
        header[name] = {"dtype": dtype, "shape": list(a.shape), "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    h = json.dumps(header).encode()
    h += b" " * ((8 - len(h) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)


def bf16_round_trip(a: np.ndarray) -> np.ndarray:
    """The values a BF16 safetensors entry holds once widened back to fp32."""
    return ((np.ascontiguousarray(a, dtype=np.float32).view(np.uint32) >> 16) << 16).view(np.float32)


def write_model_dir(path: str, shape, weights: dict, dtype: str = "F32") -> list[str]:
    from fastembed_b200 import workload as W
    os.makedirs(path, exist_ok=True)
    with open(os.path.join(path, "config.json"), "w") as f:
        json.dump(W.config_json(shape), f)
    vocab = synthetic_vocab(shape.vocab)
    with open(os.path.join(path, "vocab.txt"), "w", encoding="utf-8") as f:
        f.write("\n".join(vocab) + "\n")
    write_safetensors(os.path.join(path, "model.safetensors"), weights, dtype)
    return vocab
