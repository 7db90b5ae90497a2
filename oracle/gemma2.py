"""CPU restatement of EmbeddingGemma 2's text tower (fiber/ai
models/gemma embed.go:247-377 encode2 / encode2From, then pool, applyHead
and l2normalize, embed.go:381-475), the checker for the device path of
ai_b200/csrc/fg_model.cu (forward_v2).

TEST INFRASTRUCTURE ONLY: imported by tests/, never by the product.

Arithmetic is float64 throughout, except where the reference's own
float32 rounding is part of the result: the pre-norm folds W' = diag(g)·W
(model.go:206-222) and the RoPE tables (float64 angles stored as float32,
rope.go:36-50). Masked keys are left out of the softmax; in the reference
their additive −1e9 makes exp() flush to exactly 0 in float32, so every
query row with a visible key gets the same result. A length-0 sequence is
row 0 holding the pad id alone, what the reference's all-masked row 0
computes (its keys carry equal masks and identical values).

Parity pin: none beyond this restatement — the reference's goldens for
EmbeddingGemma 2 (testdata/eg2_*.bin) need the real checkpoint, and
transformers 5.5 here has no embedding_gemma2 class. Parity unpinned.
"""
from __future__ import annotations

import math
from typing import Dict, Optional, Sequence, Tuple

import numpy as np


def _cfg(cfg: dict) -> dict:
    t = dict(cfg["text_config"]) if cfg.get("model_type") == "embedding_gemma2" else dict(cfg)
    L = t["num_hidden_layers"]
    if not t.get("layer_types"):
        t["layer_types"] = ["full_attention" if (i + 1) % 6 == 0 else "sliding_attention" for i in range(L)]
    if t.get("per_layer_config") is None:
        t["per_layer_config"] = {f"{i:02d}": {"head_dim": 512, "num_key_value_heads": 1}
                                 for i, ty in enumerate(t["layer_types"]) if ty == "full_attention"}
    rp = t.get("rope_parameters") or {"sliding_attention": {"rope_theta": 10000.0},
                                       "full_attention": {"rope_theta": 1000000.0}}
    t["rope_parameters"] = rp
    t.setdefault("embedding_dim", 768)
    return t


def _geometry(t: dict, l: int) -> Tuple[int, int]:
    o = t["per_layer_config"].get(f"{l:02d}", t["per_layer_config"].get(str(l), {})) or {}
    return int(o.get("head_dim") or t["head_dim"]), int(o.get("num_key_value_heads") or t["num_key_value_heads"])


def _rms(x: np.ndarray, eps: float) -> np.ndarray:
    return 1.0 / np.sqrt((x * x).mean(-1, keepdims=True) + eps)


def _gelu(x: np.ndarray) -> np.ndarray:
    return 0.5 * x * (1.0 + np.tanh(math.sqrt(2.0 / math.pi) * (x + 0.044715 * x ** 3)))


def _rope_tables(base: float, T: int, D: int) -> Tuple[np.ndarray, np.ndarray]:
    half = D // 2
    inv = base ** (-np.arange(0, half, dtype=np.float64) * 2.0 / D)
    ang = np.arange(T, dtype=np.float64)[:, None] * inv[None, :]
    return np.cos(ang).astype(np.float32).astype(np.float64), np.sin(ang).astype(np.float32).astype(np.float64)


def _rope(x: np.ndarray, c: np.ndarray, s: np.ndarray) -> np.ndarray:
    """rotate-half over the last axis; x [T, heads, D], tables [T, D/2]."""
    half = x.shape[-1] // 2
    x1, x2 = x[..., :half], x[..., half:]
    cc, ss = c[:, None, :], s[:, None, :]
    return np.concatenate([x1 * cc - x2 * ss, x1 * ss + x2 * cc], axis=-1)


class Gemma2Oracle:
    """From float32 weights keyed by safetensors name, stored [out, in]."""

    def __init__(self, cfg: dict, w: Dict[str, np.ndarray], dense_tanh: Sequence[bool] = (), l2: bool = True):
        self.t = t = _cfg(cfg)
        self.w = {k: np.asarray(v, np.float32) for k, v in w.items()}
        self.dense_tanh = list(dense_tanh)
        self.l2 = l2
        H = t["hidden_size"]
        self.fold = {}
        for l in range(t["num_hidden_layers"]):
            p = f"layers.{l}."
            g_in = self.w[p + "input_layernorm.weight"]
            g_pf = self.w[p + "pre_feedforward_layernorm.weight"]
            for name, g in (("self_attn.q_proj", g_in), ("self_attn.k_proj", g_in), ("self_attn.v_proj", g_in),
                            ("mlp.gate_proj", g_pf), ("mlp.up_proj", g_pf)):
                self.fold[p + name] = (self.w[p + name + ".weight"] * g[None, :]).astype(np.float32)
        self.H = H

    def _seq(self, ids: np.ndarray) -> np.ndarray:
        """Final hidden states [T, H] of one sequence of valid ids."""
        t, w = self.t, self.w
        H, Hq, L, P = t["hidden_size"], t["num_attention_heads"], t["num_hidden_layers"], t["hidden_size_per_layer_input"]
        eps = float(t["rms_norm_eps"])
        T = len(ids)
        x = w["embed_tokens.weight"][ids].astype(np.float64) * math.sqrt(H)
        pl = (x @ w["ple.per_layer_model_projection.weight"].astype(np.float64).T) / math.sqrt(H)
        pl = pl.reshape(T, L, P)
        ple = pl * _rms(pl, eps) * w["ple.per_layer_projection_norm.weight"].astype(np.float64)
        wnd = t["sliding_window"] + 1
        pos = np.arange(T)
        for l in range(L):
            p = f"layers.{l}."
            D, Hkv = _geometry(t, l)
            sliding = t["layer_types"][l] == "sliding_attention"
            base = float(t["rope_parameters"][t["layer_types"][l]]["rope_theta"])
            f = lambda n: self.fold[p + n].astype(np.float64)  # noqa: E731
            rs = _rms(x, eps)
            q = ((x @ f("self_attn.q_proj").T) * rs).reshape(T, Hq, D)
            k = ((x @ f("self_attn.k_proj").T) * rs).reshape(T, Hkv, D)
            v = ((x @ f("self_attn.v_proj").T) * rs).reshape(T, Hkv, D)
            q = q * _rms(q, eps) * w[p + "self_attn.q_norm.weight"].astype(np.float64)
            k = k * _rms(k, eps) * w[p + "self_attn.k_norm.weight"].astype(np.float64)
            v = v * _rms(v, eps)
            c, s = _rope_tables(base, T, D)
            q, k = _rope(q, c, s), _rope(k, c, s)
            vis = np.ones((T, T), bool)
            if sliding:
                vis = np.abs(pos[:, None] - pos[None, :]) < wnd
            rep = Hq // Hkv
            att = np.empty((T, Hq, D))
            for h in range(Hq):
                sc = q[:, h, :] @ k[:, h // rep, :].T  # scores unscaled (model.go:105-109)
                sc = np.where(vis, sc, -np.inf)
                sc = np.exp(sc - sc.max(1, keepdims=True))
                att[:, h, :] = (sc / sc.sum(1, keepdims=True)) @ v[:, h // rep, :]
            o = att.reshape(T, Hq * D) @ w[p + "self_attn.o_proj.weight"].astype(np.float64).T
            x = x + o * _rms(o, eps) * w[p + "post_attention_layernorm.weight"].astype(np.float64)
            rs = _rms(x, eps)
            gate = (x @ f("mlp.gate_proj").T) * rs
            up = (x @ f("mlp.up_proj").T) * rs
            mlp = (_gelu(gate) * up) @ w[p + "mlp.down_proj.weight"].astype(np.float64).T
            x = x + mlp * _rms(mlp, eps) * w[p + "post_feedforward_layernorm.weight"].astype(np.float64)
            g = _gelu(x @ w[p + "ple_block.per_layer_input_gate.weight"].astype(np.float64).T) * ple[:, l, :]
            y = g @ w[p + "ple_block.per_layer_projection.weight"].astype(np.float64).T
            y = y * _rms(y, eps) * w[p + "ple_block.post_per_layer_input_norm.weight"].astype(np.float64)
            x = (x + y) * float(w[p + "layer_scalar"].reshape(-1)[0])
        return x * _rms(x, eps) * w["norm.weight"].astype(np.float64)

    def embed_padded(self, ids: np.ndarray, lengths: np.ndarray, dim: Optional[int] = None) -> np.ndarray:
        w = self.w
        out = []
        for b in range(ids.shape[0]):
            n = int(lengths[b])
            seq = ids[b, :n] if n > 0 else np.zeros(1, ids.dtype)
            h = self._seq(seq)
            pooled = h.mean(0)
            e = pooled @ w["embedding_projection.weight"].astype(np.float64).T
            j = 0
            while f"dense.{j}.linear.weight" in w:
                e = e @ w[f"dense.{j}.linear.weight"].astype(np.float64).T
                if j < len(self.dense_tanh) and self.dense_tanh[j]:
                    e = np.tanh(e)
                j += 1
            if dim:
                e = e[:dim]
            if self.l2:
                e = e / math.sqrt(float(e @ e) + 1e-12)
            out.append(e)
        return np.stack(out)


def from_bf16(cfg: dict, weights_bf16: Dict[str, np.ndarray]) -> Gemma2Oracle:
    from ai_b200.synthetic import bf16_to_f32

    return Gemma2Oracle(cfg, {k: bf16_to_f32(v) for k, v in weights_bf16.items()})
