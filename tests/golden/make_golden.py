"""Generates the committed golden fixtures that pin the CPU oracle.

The reference (Go) cannot be built or run here, and its own model-level
goldens (models/gemma/testdata/reference*.bin) need the real, gated
EmbeddingGemma weights. The reference validates itself against
sentence-transformers / Hugging Face at cosine 1.000000
(docs/manual/models.md:92-106, models/gemma/gemma_test.go:63-115), so this
script pins the oracle the same way: the random-init encoders of
ai_b200.synthetic are run through Hugging Face transformers'
Gemma3TextModel (use_bidirectional_attention=True, float64, eager
attention), followed by masked mean pooling, the Dense head and L2
normalisation in float64, and the embeddings are stored with the inputs.

Run here (transformers is importable in this container, not needed on the
GPU box):   python tests/golden/make_golden.py
"""
from __future__ import annotations

import hashlib
import json
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

from ai_b200 import synthetic as S  # noqa: E402

OUT = Path(__file__).resolve().parent

# name, config overrides, weight seed, norm_std, ids seed, batch lengths, T
CASES = [
    # config 1 of the benchmark: full shape, seed-0 weights (norms 0), B=8 × T=128
    ("c1", {}, 0, 0.0, 0, [128] * 8, 128),
    # sliding and global layers with a sequence longer than the window
    # (bound 257), padding, non-zero norm weights
    ("window", {"num_hidden_layers": 6, "vocab_size": 4096}, 7, 0.1, 8, [300, 280, 40, 1], 300),
    # ragged short batch on the full vocabulary, non-zero norms, 3 layers
    ("ragged", {"num_hidden_layers": 3}, 11, 0.05, 12, [33, 17, 64, 5, 2], 64),
]


def weights_digest(w) -> str:
    h = hashlib.sha256()
    for k in sorted(w):
        h.update(k.encode())
        h.update(np.ascontiguousarray(w[k]).tobytes())
    return h.hexdigest()


def hf_embed(cfg: dict, w: dict, ids: np.ndarray, lengths: np.ndarray) -> np.ndarray:
    import torch
    from transformers import Gemma3TextConfig, Gemma3TextModel

    hcfg = Gemma3TextConfig(
        vocab_size=cfg["vocab_size"], hidden_size=cfg["hidden_size"],
        intermediate_size=cfg["intermediate_size"], num_hidden_layers=cfg["num_hidden_layers"],
        num_attention_heads=cfg["num_attention_heads"],
        num_key_value_heads=cfg["num_key_value_heads"], head_dim=cfg["head_dim"],
        hidden_activation="gelu_pytorch_tanh", max_position_embeddings=cfg["max_position_embeddings"],
        rms_norm_eps=cfg["rms_norm_eps"], query_pre_attn_scalar=cfg["query_pre_attn_scalar"],
        sliding_window=cfg["sliding_window"], use_bidirectional_attention=True,
        rope_theta=cfg["rope_theta"], rope_local_base_freq=cfg["rope_local_base_freq"],
        attn_implementation="eager", pad_token_id=0, bos_token_id=2, eos_token_id=1)
    model = Gemma3TextModel(hcfg).to(torch.float64).eval()
    sd = {k: torch.from_numpy(S.bf16_to_f32(v).astype(np.float64))
          for k, v in w.items() if not k.startswith("dense.")}
    missing, unexpected = model.load_state_dict(sd, strict=False)
    assert not unexpected, unexpected
    assert all("rotary" in m for m in missing), missing
    # One unpadded sequence per call: Hugging Face's eager attention turns a
    # padded query row with no visible key into NaN, which then leaks into
    # valid rows through 0·NaN; an unpadded run is the padding-free truth.
    B, T = ids.shape
    pooled = []
    with torch.no_grad():
        for b in range(B):
            n = max(int(lengths[b]), 1)
            seq = ids[b, :n] if lengths[b] > 0 else np.zeros(1, ids.dtype)
            h = model(input_ids=torch.from_numpy(seq[None].astype(np.int64))).last_hidden_state
            pooled.append(h[0].numpy().mean(0))
    pooled = np.stack(pooled)
    x = pooled
    j = 0
    while f"dense.{j}.linear.weight" in w:
        x = x @ S.bf16_to_f32(w[f"dense.{j}.linear.weight"]).astype(np.float64).T
        j += 1
    return x / np.sqrt((x * x).sum(-1, keepdims=True) + 1e-12)


def main():
    import torch

    torch.set_num_threads(8)
    manifest = {}
    for name, over, seed, norm_std, ids_seed, lens, T in CASES:
        cfg = dict(S.EMBEDDINGGEMMA_300M)
        cfg.update(over)
        w = S.make_weights(cfg, seed=seed, norm_std=norm_std)
        B = len(lens)
        ids = S.make_ids(B, T, ids_seed, cfg["vocab_size"])
        lengths = np.array(lens, dtype=np.int32)
        emb = hf_embed(cfg, w, ids, lengths)
        np.savez_compressed(OUT / f"{name}.npz", ids=ids, lengths=lengths, hf=emb)
        manifest[name] = {"config": over, "seed": seed, "norm_std": norm_std, "ids_seed": ids_seed,
                          "weights_sha256": weights_digest(w)}
        print(name, emb.shape, flush=True)
    (OUT / "manifest.json").write_text(json.dumps(manifest, indent=1))


if __name__ == "__main__":
    main()
