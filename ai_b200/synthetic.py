"""Seeded synthetic model and inputs of the benchmark configurations.

No network means no checkpoint: the encoder is EmbeddingGemma-300m-shaped
with random-init weights, drawn with ``numpy.random.default_rng(seed)`` in a
fixed order (``weight_specs``), ~N(0, 0.02²), rounded to bfloat16
(round-to-nearest-even) and stored as bfloat16, so every implementation
reads bit-identical weights. RMSNorm weights are 0 (so 1 + w = 1) unless
``norm_std`` asks for non-zero ones. Token ids come from their own seeded
generators, BOS = 2 first, the rest uniform in [3, vocab).

Also here: a minimal safetensors reader/writer with BF16 support (the
reference's reader widens BF16 exactly, safetensors/convert.go:31-38), and
``write_model_dir`` for the Hugging Face / sentence-transformers layout
``gemma.Load`` reads (config.json, model.safetensors, modules.json, Dense
module directories).
"""
from __future__ import annotations

import json
import struct
from pathlib import Path
from typing import Dict, Iterable, List, Tuple

import numpy as np

# EmbeddingGemma-300m text encoder shape (query_pre_attn_scalar and
# rms_norm_eps are the checkpoint's values).
EMBEDDINGGEMMA_300M = {
    "architectures": ["Gemma3TextModel"],
    "model_type": "gemma3_text",
    "hidden_size": 768,
    "intermediate_size": 1152,
    "num_hidden_layers": 24,
    "num_attention_heads": 3,
    "num_key_value_heads": 1,
    "head_dim": 256,
    "vocab_size": 262144,
    "sliding_window": 512,
    "rope_theta": 1000000.0,
    "rope_local_base_freq": 10000.0,
    "query_pre_attn_scalar": 256,
    "rms_norm_eps": 1e-06,
    "hidden_activation": "gelu_pytorch_tanh",
    "use_bidirectional_attention": True,
    "max_position_embeddings": 2048,
    "attention_bias": False,
    "attn_logit_softcapping": None,
    "final_logit_softcapping": None,
    "bos_token_id": 2,
    "eos_token_id": 1,
    "pad_token_id": 0,
}
HEAD_DIMS = [(768, 3072), (3072, 768)]  # Dense 768→3072→768, Identity activation
BOS = 2


def bf16_round(x: np.ndarray) -> np.ndarray:
    """float32 → bfloat16 bits (uint16), round to nearest even."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    r = (u + np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))) >> np.uint32(16)
    return r.astype(np.uint16)


def bf16_to_f32(b: np.ndarray) -> np.ndarray:
    """bfloat16 bits → float32, exact (the top half of a float32)."""
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << np.uint32(16)).view(np.float32)


def weight_specs(cfg: dict, head=HEAD_DIMS) -> List[Tuple[str, Tuple[int, ...], str]]:
    """(name, shape, kind) in generation order; kind 'w' = N(0,0.02²), 'n' = norm."""
    H, F, D = cfg["hidden_size"], cfg["intermediate_size"], cfg["head_dim"]
    Hq, Hkv, V = cfg["num_attention_heads"], cfg["num_key_value_heads"], cfg["vocab_size"]
    specs = [("embed_tokens.weight", (V, H), "w")]
    for l in range(cfg["num_hidden_layers"]):
        p = f"layers.{l}."
        specs += [
            (p + "self_attn.q_proj.weight", (Hq * D, H), "w"),
            (p + "self_attn.k_proj.weight", (Hkv * D, H), "w"),
            (p + "self_attn.v_proj.weight", (Hkv * D, H), "w"),
            (p + "self_attn.o_proj.weight", (H, Hq * D), "w"),
            (p + "mlp.gate_proj.weight", (F, H), "w"),
            (p + "mlp.up_proj.weight", (F, H), "w"),
            (p + "mlp.down_proj.weight", (H, F), "w"),
            (p + "input_layernorm.weight", (H,), "n"),
            (p + "post_attention_layernorm.weight", (H,), "n"),
            (p + "pre_feedforward_layernorm.weight", (H,), "n"),
            (p + "post_feedforward_layernorm.weight", (H,), "n"),
            (p + "self_attn.q_norm.weight", (D,), "n"),
            (p + "self_attn.k_norm.weight", (D,), "n"),
        ]
    specs.append(("norm.weight", (H,), "n"))
    for j, (i, o) in enumerate(head):
        specs.append((f"dense.{j}.linear.weight", (o, i), "w"))
    return specs


def make_weights(cfg: dict = EMBEDDINGGEMMA_300M, seed: int = 0, norm_std: float = 0.0,
                 head=HEAD_DIMS) -> Dict[str, np.ndarray]:
    """Random-init weights as bfloat16 bits (uint16 arrays), keyed by name.

    Matrices are drawn in ``weight_specs`` order from default_rng(seed).
    Norm weights are 0, or, when norm_std > 0, drawn from a second
    generator default_rng(seed + 1000) ~N(0, norm_std²) — zero norms hide
    (1 + w) and fold mistakes, so tests use both.
    """
    rng = np.random.default_rng(seed)
    nrng = np.random.default_rng(seed + 1000)
    out = {}
    for name, shape, kind in weight_specs(cfg, head):
        if kind == "w":
            x = rng.standard_normal(shape, dtype=np.float32)
            x *= np.float32(0.02)
        elif norm_std > 0:
            x = nrng.standard_normal(shape, dtype=np.float32) * np.float32(norm_std)
        else:
            x = np.zeros(shape, dtype=np.float32)
        out[name] = bf16_round(x)
    return out


def make_weights_f32(cfg: dict = EMBEDDINGGEMMA_300M, seed: int = 0, norm_std: float = 0.0,
                     head=HEAD_DIMS) -> Dict[str, np.ndarray]:
    """The same draws as ``make_weights`` kept in float32, not rounded to
    bfloat16: a checkpoint stored in fp32 (a fine-tuned or re-saved model),
    whose projections have no exact fp16 form and carry TF32 low parts."""
    rng = np.random.default_rng(seed)
    nrng = np.random.default_rng(seed + 1000)
    out = {}
    for name, shape, kind in weight_specs(cfg, head):
        if kind == "w":
            x = rng.standard_normal(shape, dtype=np.float32)
            x *= np.float32(0.02)
        elif norm_std > 0:
            x = nrng.standard_normal(shape, dtype=np.float32) * np.float32(norm_std)
        else:
            x = np.zeros(shape, dtype=np.float32)
        out[name] = x
    return out


# EmbeddingGemma 2's text tower, shaped as the reference's config test
# (models/gemma/gemma2_test.go TestConfig2): 12 layers of width 512, layers 5
# and 11 global with 512-wide heads and one KV head, per-layer inputs of 512,
# a 768-wide embedding projection.
EMBEDDINGGEMMA2_TEXT = {
    "hidden_size": 512,
    "intermediate_size": 2048,
    "num_hidden_layers": 12,
    "num_attention_heads": 4,
    "num_key_value_heads": 2,
    "head_dim": 256,
    "vocab_size": 262144,
    "sliding_window": 512,
    "rms_norm_eps": 1e-06,
    "hidden_activation": "gelu_pytorch_tanh",
    "hidden_size_per_layer_input": 512,
    "embedding_dim": 768,
    "max_position_embeddings": 8192,
    "per_layer_config": {"05": {"head_dim": 512, "num_key_value_heads": 1},
                         "11": {"head_dim": 512, "num_key_value_heads": 1}},
    "rope_parameters": {"full_attention": {"rope_theta": 1000000.0, "rope_type": "default"},
                        "sliding_attention": {"rope_theta": 10000.0, "rope_type": "default"}},
}


def eg2_config(text: dict = EMBEDDINGGEMMA2_TEXT) -> dict:
    """An embedding_gemma2 config.json (text tower only)."""
    return {"model_type": "embedding_gemma2", "text_config": dict(text)}


def eg2_small_config(layers: int = 3, hidden: int = 256, vocab: int = 4096, window: int = 48,
                     full=(1,), ple: int = 128, emb: int = 192) -> dict:
    """A small EmbeddingGemma 2 for tests: `full` layers global with 512-wide
    heads and one KV head, the others sliding (radius `window`) with 256-wide
    heads and two KV heads."""
    t = dict(EMBEDDINGGEMMA2_TEXT)
    t.update({"hidden_size": hidden, "intermediate_size": 512, "num_hidden_layers": layers,
              "vocab_size": vocab, "sliding_window": window, "hidden_size_per_layer_input": ple,
              "embedding_dim": emb,
              "layer_types": ["full_attention" if l in full else "sliding_attention" for l in range(layers)],
              "per_layer_config": {f"{l:02d}": {"head_dim": 512, "num_key_value_heads": 1} for l in full}})
    return eg2_config(t)


def _eg2_geometry(t: dict, l: int) -> Tuple[int, int]:
    o = (t.get("per_layer_config") or {}).get(f"{l:02d}", {})
    return int(o.get("head_dim") or t["head_dim"]), int(o.get("num_key_value_heads") or t["num_key_value_heads"])


def weight_specs_eg2(cfg: dict, head=()) -> List[Tuple[str, Tuple[int, ...], str]]:
    """EmbeddingGemma 2's text-tower weights (model.go:142-205): kind 'w' =
    N(0,0.02²), 'n' = a norm that multiplies by its weight (1 + noise),
    'q' = a q/k norm, 's' = the layer scalar."""
    t = cfg["text_config"]
    H, F, Hq, V = t["hidden_size"], t["intermediate_size"], t["num_attention_heads"], t["vocab_size"]
    L, P, E = t["num_hidden_layers"], t["hidden_size_per_layer_input"], t.get("embedding_dim") or 768
    specs = [("embed_tokens.weight", (V, H), "w")]
    for l in range(L):
        D, Hkv = _eg2_geometry(t, l)
        p = f"layers.{l}."
        specs += [
            (p + "self_attn.q_proj.weight", (Hq * D, H), "w"),
            (p + "self_attn.k_proj.weight", (Hkv * D, H), "w"),
            (p + "self_attn.v_proj.weight", (Hkv * D, H), "w"),
            (p + "self_attn.o_proj.weight", (H, Hq * D), "w"),
            (p + "mlp.gate_proj.weight", (F, H), "w"),
            (p + "mlp.up_proj.weight", (F, H), "w"),
            (p + "mlp.down_proj.weight", (H, F), "w"),
            (p + "ple_block.per_layer_input_gate.weight", (P, H), "w"),
            (p + "ple_block.per_layer_projection.weight", (H, P), "w"),
            (p + "input_layernorm.weight", (H,), "n"),
            (p + "post_attention_layernorm.weight", (H,), "n"),
            (p + "pre_feedforward_layernorm.weight", (H,), "n"),
            (p + "post_feedforward_layernorm.weight", (H,), "n"),
            (p + "self_attn.q_norm.weight", (D,), "q"),
            (p + "self_attn.k_norm.weight", (D,), "q"),
            (p + "ple_block.post_per_layer_input_norm.weight", (H,), "n"),
            (p + "layer_scalar", (1,), "s"),
        ]
    specs += [("norm.weight", (H,), "n"),
              ("ple.per_layer_model_projection.weight", (L * P, H), "w"),
              ("ple.per_layer_projection_norm.weight", (P,), "n"),
              ("embedding_projection.weight", (E, H), "w")]
    for j, (i, o) in enumerate(head):
        specs.append((f"dense.{j}.linear.weight", (o, i), "w"))
    return specs


def make_weights_eg2(cfg: dict, seed: int = 0, norm_std: float = 0.1, head=()) -> Dict[str, np.ndarray]:
    """Random-init EmbeddingGemma 2 weights as bfloat16 bits: matrices
    ~N(0, 0.02²) from default_rng(seed) in weight_specs_eg2 order; norms
    1 + N(0, norm_std²), q/k norms D^(-1/4)·(1 + N(0, norm_std²)) and layer
    scalars uniform in [0.5, 1.5) from default_rng(seed + 1000).

    The scores are not scaled in this architecture (model.go:105-109), so a
    trained model's q/k norm weights keep q·k of order one; unit q/k gains
    would give logits of order √D, a near-argmax softmax, and a random
    model that amplifies every rounding difference by orders of magnitude.
    D^(-1/4) on each side restores logits of order one."""
    rng = np.random.default_rng(seed)
    nrng = np.random.default_rng(seed + 1000)
    out = {}
    for name, shape, kind in weight_specs_eg2(cfg, head):
        if kind == "w":
            x = rng.standard_normal(shape, dtype=np.float32) * np.float32(0.02)
        elif kind == "n":
            x = np.float32(1) + nrng.standard_normal(shape, dtype=np.float32) * np.float32(norm_std)
        elif kind == "q":
            x = (np.float32(1) + nrng.standard_normal(shape, dtype=np.float32) * np.float32(norm_std)) \
                * np.float32(shape[0] ** -0.25)
        else:
            x = nrng.uniform(0.5, 1.5, shape).astype(np.float32)
        out[name] = bf16_round(x.astype(np.float32))
    return out


def make_ids(batch: int, seq: int, seed: int, vocab: int = 262144) -> np.ndarray:
    """[batch, seq] int32 ids: BOS first, the rest uniform in [3, vocab)."""
    rng = np.random.default_rng(seed)
    ids = np.empty((batch, seq), dtype=np.int32)
    ids[:, 0] = BOS
    if seq > 1:
        ids[:, 1:] = rng.integers(3, vocab, size=(batch, seq - 1), dtype=np.int64)
    return ids


def make_ragged(n: int, lo: int, hi: int, seed: int, vocab: int = 262144):
    """n sequences, lengths uniform in [lo, hi] (both inclusive), ids as in
    make_ids; returns (list of int32 arrays, lengths int32 array)."""
    rng = np.random.default_rng(seed)
    lengths = rng.integers(lo, hi + 1, size=n, dtype=np.int64).astype(np.int32)
    seqs = []
    for L in lengths:
        s = np.empty(int(L), dtype=np.int32)
        s[0] = BOS
        if L > 1:
            s[1:] = rng.integers(3, vocab, size=int(L) - 1, dtype=np.int64)
        seqs.append(s)
    return seqs, lengths


def small_config(layers: int = 2, vocab: int = 4096, **over) -> dict:
    """The same architecture with fewer layers and a smaller vocabulary, for
    tests that run the CPU oracle at many shapes."""
    c = dict(EMBEDDINGGEMMA_300M)
    c["num_hidden_layers"] = layers
    c["vocab_size"] = vocab
    c.update(over)
    return c


# ----------------------------------------------------------------- safetensors
_DT = {"F32": np.float32, "F16": np.float16, "BF16": np.uint16, "F64": np.float64,
       "I32": np.int32, "I64": np.int64}


def read_safetensors(path) -> Dict[str, Tuple[str, np.ndarray]]:
    """name → (dtype string, array); BF16 stays as uint16 bits."""
    data = Path(path).read_bytes()
    (n,) = struct.unpack("<Q", data[:8])
    header = json.loads(data[8:8 + n])
    base = 8 + n
    out = {}
    for name, info in header.items():
        if name == "__metadata__":
            continue
        dt = info["dtype"]
        if dt not in _DT:
            raise ValueError(f"safetensors: dtype {dt} of {name} not supported")
        s, e = info["data_offsets"]
        arr = np.frombuffer(data, dtype=_DT[dt], count=(e - s) // np.dtype(_DT[dt]).itemsize,
                            offset=base + s).reshape(info["shape"])
        out[name] = (dt, arr)
    return out


def write_safetensors(path, tensors: Dict[str, Tuple[str, np.ndarray]]) -> None:
    header = {}
    off = 0
    blobs = []
    for name, (dt, arr) in tensors.items():
        b = np.ascontiguousarray(arr).tobytes()
        header[name] = {"dtype": dt, "shape": list(arr.shape), "data_offsets": [off, off + len(b)]}
        off += len(b)
        blobs.append(b)
    hj = json.dumps(header).encode()
    hj += b" " * ((8 - len(hj) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(hj)))
        f.write(hj)
        for b in blobs:
            f.write(b)


def write_model_dir(d, cfg: dict, weights: Dict[str, np.ndarray], head=HEAD_DIMS) -> Path:
    """Writes the sentence-transformers layout gemma.Load reads."""
    d = Path(d)
    d.mkdir(parents=True, exist_ok=True)
    (d / "config.json").write_text(json.dumps(cfg, indent=1))
    body = {k: ("BF16", v) for k, v in weights.items() if not k.startswith("dense.")}
    write_safetensors(d / "model.safetensors", body)
    modules = [{"idx": 0, "name": "0", "path": "",
                "type": "sentence_transformers.models.Transformer"},
               {"idx": 1, "name": "1", "path": "1_Pooling",
                "type": "sentence_transformers.models.Pooling"}]
    (d / "1_Pooling").mkdir(exist_ok=True)
    (d / "1_Pooling" / "config.json").write_text(json.dumps(
        {"word_embedding_dimension": cfg["hidden_size"], "pooling_mode_mean_tokens": True,
         "pooling_mode_cls_token": False, "pooling_mode_lasttoken": False,
         "include_prompt": True}))
    for j, (i, o) in enumerate(head):
        sub = f"{2 + j}_Dense"
        (d / sub).mkdir(exist_ok=True)
        (d / sub / "config.json").write_text(json.dumps(
            {"in_features": i, "out_features": o, "bias": False,
             "activation_function": "torch.nn.modules.linear.Identity"}))
        write_safetensors(d / sub / "model.safetensors",
                          {"linear.weight": ("BF16", weights[f"dense.{j}.linear.weight"])})
        modules.append({"idx": 2 + j, "name": str(2 + j), "path": sub,
                        "type": "sentence_transformers.models.Dense"})
    modules.append({"idx": 2 + len(head), "name": str(2 + len(head)),
                    "path": f"{2 + len(head)}_Normalize",
                    "type": "sentence_transformers.models.Normalize"})
    (d / "modules.json").write_text(json.dumps(modules, indent=1))
    return d
