"""ctypes binding of the CPU oracle (oracle/libfgoracle.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, by __graft_entry__.smoke()
as the checker, and by bench.py's cpu_baseline leg. The product
(ai_b200/) never imports it. Build with ``make -C oracle``.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path
from typing import Dict, Optional

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "libfgoracle.so"
F64, F32 = 0, 1
MAX_DENSE = 4

_fp = C.POINTER(C.c_float)
_fpp = C.POINTER(_fp)


class OrcConfig(C.Structure):
    _fields_ = [
        ("hidden", C.c_int), ("ffn", C.c_int), ("layers", C.c_int), ("heads", C.c_int),
        ("kv_heads", C.c_int), ("head_dim", C.c_int), ("vocab", C.c_int), ("window", C.c_int),
        ("eps", C.c_float), ("attn_scale", C.c_float),
        ("sliding", C.POINTER(C.c_int)), ("rope_base", C.POINTER(C.c_double)),
        ("num_dense", C.c_int),
        ("dense_in", C.c_int * MAX_DENSE), ("dense_out", C.c_int * MAX_DENSE),
        ("dense_tanh", C.c_int * MAX_DENSE), ("l2", C.c_int),
    ]


class OrcWeights(C.Structure):
    _fields_ = [
        ("embed", _fp),
        ("in_norm", _fpp), ("post_attn_norm", _fpp), ("pre_ffn_norm", _fpp),
        ("post_ffn_norm", _fpp), ("q_norm", _fpp), ("k_norm", _fpp),
        ("wq", _fpp), ("wk", _fpp), ("wv", _fpp), ("wo", _fpp),
        ("wgate", _fpp), ("wup", _fpp), ("wdown", _fpp),
        ("final_norm", _fp), ("dense", _fp * MAX_DENSE),
    ]


_lib = None


def set_fast_kernels(on: bool) -> None:
    """Float32 mode: packed AVX-512 kernels (default) or the simple loops;
    bit for bit the same results."""
    lib().orc_set_fast_kernels(1 if on else 0)


def build() -> Path:
    """Builds libfgoracle.so with the committed Makefile (idempotent)."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not LIB.exists():
            build()
        h = C.CDLL(str(LIB))
        h.orc_embed.argtypes = [C.POINTER(OrcConfig), C.POINTER(OrcWeights), C.c_void_p, C.c_void_p,
                                C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_void_p]
        h.orc_embed.restype = C.c_int
        h.orc_matmul_fused.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int,
                                       C.c_void_p, C.c_void_p, C.c_int, C.c_void_p, C.c_void_p,
                                       C.c_int, C.c_void_p]
        h.orc_attention_head.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int,
                                         C.c_int, C.c_int, C.c_float, C.c_int, C.c_void_p]
        h.orc_rmsnorm.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_float, C.c_int,
                                  C.c_void_p]
        h.orc_rope.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_double, C.c_void_p,
                               C.c_void_p]
        h.orc_window_mask.argtypes = [C.c_int, C.c_int, C.c_void_p]
        h.orc_padding_mask.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_void_p]
        for n in ("orc_exp_ref", "orc_tanh_ref", "orc_gelu_ref"):
            getattr(h, n).argtypes = [C.c_void_p, C.c_int, C.c_void_p]
        h.orc_set_fast_kernels.argtypes = [C.c_int]
        h.orc_set_fast_kernels.restype = None
        _lib = h
    return _lib


def _p(a: Optional[np.ndarray]):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


class OracleModel:
    """The reference encoder on the CPU, from float32 weights keyed by the
    safetensors names (raw, as stored: [out, in] projections, w not 1+w)."""

    def __init__(self, cfg: dict, weights_f32: Dict[str, np.ndarray], dense_tanh=(), l2=True):
        self.cfg = cfg
        L = cfg["num_hidden_layers"]
        sw = cfg.get("sliding_window", 0)
        window = (sw // 2 + 1) if cfg.get("use_bidirectional_attention") else sw
        pattern = cfg.get("sliding_window_pattern") or 6
        types = cfg.get("layer_types") or ["full_attention" if (i + 1) % pattern == 0
                                           else "sliding_attention" for i in range(L)]
        sliding = [1 if t == "sliding_attention" else 0 for t in types]
        loc = cfg.get("rope_local_base_freq") or 10000.0
        glob = cfg.get("rope_theta") or 10000.0
        bases = [loc if s else glob for s in sliding]
        self._keep = []
        w = {k: _f32(v) for k, v in weights_f32.items()}
        self._keep.append(w)
        self._sliding = (C.c_int * L)(*sliding)
        self._bases = (C.c_double * L)(*bases)
        c = OrcConfig()
        c.hidden, c.ffn, c.layers = cfg["hidden_size"], cfg["intermediate_size"], L
        c.heads, c.kv_heads = cfg["num_attention_heads"], cfg["num_key_value_heads"]
        c.head_dim, c.vocab = cfg["head_dim"], cfg["vocab_size"]
        c.window = window if sw > 0 else 0
        c.eps = cfg["rms_norm_eps"]
        c.attn_scale = float(np.float32(1.0 / np.sqrt(cfg["query_pre_attn_scalar"])))
        c.sliding, c.rope_base = self._sliding, self._bases
        j = 0
        while f"dense.{j}.linear.weight" in w:
            o, i = w[f"dense.{j}.linear.weight"].shape
            c.dense_in[j], c.dense_out[j] = i, o
            c.dense_tanh[j] = int(j < len(dense_tanh) and dense_tanh[j])
            j += 1
        c.num_dense = j
        c.l2 = int(l2)
        self.c = c
        self.dim = c.dense_out[j - 1] if j else c.hidden

        def arr(name):
            return w[name].ctypes.data_as(_fp)

        def per_layer(suffix):
            a = (_fp * L)(*[arr(f"layers.{l}.{suffix}") for l in range(L)])
            self._keep.append(a)
            return a

        ws = OrcWeights()
        ws.embed = arr("embed_tokens.weight")
        ws.in_norm = per_layer("input_layernorm.weight")
        ws.post_attn_norm = per_layer("post_attention_layernorm.weight")
        ws.pre_ffn_norm = per_layer("pre_feedforward_layernorm.weight")
        ws.post_ffn_norm = per_layer("post_feedforward_layernorm.weight")
        ws.q_norm = per_layer("self_attn.q_norm.weight")
        ws.k_norm = per_layer("self_attn.k_norm.weight")
        ws.wq = per_layer("self_attn.q_proj.weight")
        ws.wk = per_layer("self_attn.k_proj.weight")
        ws.wv = per_layer("self_attn.v_proj.weight")
        ws.wo = per_layer("self_attn.o_proj.weight")
        ws.wgate = per_layer("mlp.gate_proj.weight")
        ws.wup = per_layer("mlp.up_proj.weight")
        ws.wdown = per_layer("mlp.down_proj.weight")
        ws.final_norm = arr("norm.weight")
        for i in range(j):
            ws.dense[i] = arr(f"dense.{i}.linear.weight")
        self.ws = ws

    def embed_padded(self, ids: np.ndarray, lengths: np.ndarray, dim: Optional[int] = None,
                     mode: int = F64, threads: int = 0) -> np.ndarray:
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        lengths = np.ascontiguousarray(lengths, dtype=np.int32)
        B, T = ids.shape
        dim = self.dim if dim is None else dim
        out = np.empty((B, dim), dtype=np.float32)
        rc = lib().orc_embed(C.byref(self.c), C.byref(self.ws), _p(ids), _p(lengths), B, T, dim,
                             mode, threads, _p(out))
        if rc != 0:
            raise RuntimeError("oracle: orc_embed failed")
        return out


def from_bf16(cfg: dict, weights_bf16: Dict[str, np.ndarray]) -> OracleModel:
    from ai_b200.synthetic import bf16_to_f32

    return OracleModel(cfg, {k: bf16_to_f32(v) for k, v in weights_bf16.items()})


# ------------------------------------------------------------- op-level
def matmul_fused(x, w, bias=None, row_scale=None, act=0, mul=None, residual=None, mode=F64):
    x, w = _f32(x), _f32(w)
    m, k = x.shape
    n = w.shape[1]
    out = np.empty((m, n), np.float32)
    args = [None if a is None else _f32(a) for a in (bias, row_scale, mul, residual)]
    lib().orc_matmul_fused(_p(x), _p(w), m, k, n, _p(args[0]), _p(args[1]), act, _p(args[2]),
                           _p(args[3]), mode, _p(out))
    return out


def attention_head(q, k, v, mask, scale, mode=F64):
    q, k, v = _f32(q), _f32(k), _f32(v)
    T, D = q.shape
    S = k.shape[0]
    m = None if mask is None else _f32(mask)
    out = np.empty((T, D), np.float32)
    lib().orc_attention_head(_p(q), _p(k), _p(v), _p(m), T, S, D, scale, mode, _p(out))
    return out


def rmsnorm(x, g, eps, mode=F64):
    x, g = _f32(x), _f32(g)
    n = x.shape[-1]
    out = np.empty_like(x)
    lib().orc_rmsnorm(_p(x), x.size // n, n, _p(g), eps, mode, _p(out))
    return out


def rope(x, base, positions):
    x = _f32(x)
    T, D = x.shape[-2], x.shape[-1]
    pos = np.ascontiguousarray(positions, dtype=np.int32)
    out = np.empty_like(x)
    lib().orc_rope(_p(x), x.size // D, T, D, float(base), _p(pos), _p(out))
    return out


def window_mask(n, w):
    out = np.empty((n, n), np.float32)
    lib().orc_window_mask(n, w, _p(out))
    return out


def padding_mask(lengths, n):
    l = np.ascontiguousarray(lengths, dtype=np.int32)
    out = np.empty((len(l), n), np.float32)
    lib().orc_padding_mask(_p(l), len(l), n, _p(out))
    return out


def exp_ref(x):
    x = _f32(x)
    out = np.empty_like(x)
    lib().orc_exp_ref(_p(x), x.size, _p(out))
    return out


def tanh_ref(x):
    x = _f32(x)
    out = np.empty_like(x)
    lib().orc_tanh_ref(_p(x), x.size, _p(out))
    return out


def gelu_ref(x):
    x = _f32(x)
    out = np.empty_like(x)
    lib().orc_gelu_ref(_p(x), x.size, _p(out))
    return out
