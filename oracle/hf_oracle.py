"""Oracle for the Qwen3- and Gemma3-shaped encoders: HF transformers on the CPU in FP32.

Test infrastructure only (tests/, the golden-fixture generator).  These model families
are not in the reference, so parity for them is pinned against the model definitions
in transformers (Qwen3Model, Gemma3TextModel with bidirectional attention), not against
the reference: each sentence runs alone and unpadded (equivalent to masking a padded
batch), the final-norm hidden states are pooled (last token for Qwen3, mean for
Gemma3) and L2-normalised.
"""
from __future__ import annotations

import numpy as np


def build(shape, weights: dict):
    import torch
    from fastembed_b200 import workload as W
    kw = W.rms_hf_config(shape)
    if shape.family == "qwen3":
        from transformers import Qwen3Config, Qwen3Model
        model = Qwen3Model(Qwen3Config(**kw))
    else:
        from transformers import Gemma3TextConfig, Gemma3TextModel
        model = Gemma3TextModel(Gemma3TextConfig(**kw))
    sd = {k: torch.from_numpy(np.ascontiguousarray(v)) for k, v in weights.items()}
    missing, unexpected = model.load_state_dict(sd, strict=False)
    missing = [m for m in missing if not m.endswith("rotary_emb.inv_freq")]
    if missing or unexpected:
        raise ValueError(f"weights do not match the model: missing {missing}, unexpected {unexpected}")
    return model.float().eval()


def embed(shape, weights: dict, ids: np.ndarray, lengths: np.ndarray) -> np.ndarray:
    """[B, hidden] L2-normalised sentence embeddings, FP32."""
    import torch
    model = build(shape, weights)
    out = np.zeros((lengths.size, shape.hidden), np.float32)
    with torch.no_grad():
        for b, L in enumerate(lengths):
            L = int(L)
            if L == 0:
                continue
            x = torch.from_numpy(ids[b:b + 1, :L].astype(np.int64))
            h = model(input_ids=x).last_hidden_state[0]
            v = h[-1] if shape.pooling == "last" else h.mean(0)
            out[b] = (v / v.norm()).numpy()
    return out
