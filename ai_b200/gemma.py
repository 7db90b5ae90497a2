"""Host-side mirror of fiber/ai's ``models/gemma`` for the EmbeddingGemma encoder.

Same names, argument meaning and error behaviour as the reference, with
the compute in libfgemma (C ABI, include/fgemma.h):

- ``LoadConfig(dir)``  — models/gemma/config.go:153-245 (Gemma 3 encoders;
  the EmbeddingGemma 2 variant is outside this path and is refused);
- ``Config.window() / is_sliding(l) / rope_base(l)`` — config.go:331-362;
- ``Load(dir, *options)`` — model.go:76-232 and the head (model.go:236-310):
  reads config.json, the weight safetensors (BF16/F16/F32, widened
  exactly), modules.json and the Dense modules, and hands the weights to
  ``fg_model_set_weight`` / ``fg_model_finalize`` (which apply the (1+w)
  norms and the pre-norm folds on the device side);
- ``Model.embed_batch(ids)`` — (*Model).embedBatch (embed.go:118-157):
  right-pads with id 0 and embeds one batch;
- ``Model.embed_ids(seqs, Dim=)`` — (*Model).Embed (embed.go:15-80) from
  token ids: truncation to MaxTokens, stable length sort (sortIndex,
  model.go:412-423) and greedy batches under the padded-token budget
  ``maxLen·(n+1) ≤ BatchTokens``; results in input order. (The tokenizer is
  the reference's own, reused as-is on the host; it is not part of this
  package.)
- Options ``MaxTokens``, ``BatchTokens``, ``Threads`` (model.go:352-359).

Errors: model-level calls raise ``GemmaError`` where the reference returns
an ``error`` (e.g. "gemma: Dim(%d) outside 1..%d").
"""
from __future__ import annotations

import ctypes as C
import json
import math
from dataclasses import dataclass, field
from pathlib import Path
from typing import Callable, Dict, List, Optional, Sequence, Tuple

import numpy as np

from . import _lib
from ._lib import PREC_SPLIT, PREC_SPLIT_TF32, PREC_TF32  # noqa: F401
from .synthetic import read_safetensors


class GemmaError(RuntimeError):
    """An error the reference's model functions return."""


# ------------------------------------------------------------------ config
@dataclass
class Config:
    hidden_size: int = 0
    intermediate_size: int = 0
    num_hidden_layers: int = 0
    num_attention_heads: int = 0
    num_key_value_heads: int = 0
    head_dim: int = 0
    vocab_size: int = 0
    sliding_window: int = 0
    sliding_window_pattern: int = 0
    layer_types: List[str] = field(default_factory=list)
    rope_theta: float = 0.0
    rope_local_base_freq: float = 0.0
    query_pre_attn_scalar: float = 0.0
    rms_norm_eps: float = 0.0
    hidden_activation: str = ""
    use_bidirectional_attention: bool = False
    max_position_embeddings: int = 0
    rope_scaling: object = None
    # EmbeddingGemma 2 only (config.go:38-45): variant 2, else 0
    variant: int = 0
    hidden_size_per_layer_input: int = 0
    embedding_dim: int = 0
    per_layer_config: Optional[dict] = None
    rope_parameters: Optional[dict] = None

    def window(self) -> int:
        """Attend when |i − j| < window() (config.go:331-339). EmbeddingGemma 2
        configures an inclusive radius, so its bound is one more."""
        if self.variant == 2:
            return self.sliding_window + 1
        if self.use_bidirectional_attention:
            return self.sliding_window // 2 + 1
        return self.sliding_window

    def is_sliding(self, l: int) -> bool:
        return self.layer_types[l] == "sliding_attention"

    def _override(self, l: int) -> dict:
        pl = self.per_layer_config or {}
        return pl.get(f"{l:02d}", pl.get(str(l), {})) or {}

    def head_dim_of(self, l: int) -> int:
        """Config.headDim(l) (config.go:314-320)."""
        return int(self._override(l).get("head_dim") or self.head_dim)

    def kv_heads_of(self, l: int) -> int:
        """Config.kvHeads(l) (config.go:322-328)."""
        return int(self._override(l).get("num_key_value_heads") or self.num_key_value_heads)

    def rope_base(self, l: int) -> float:
        """Local base on sliding layers, global theta otherwise (config.go:346-362);
        EmbeddingGemma 2 reads rope_parameters per layer type."""
        if self.variant == 2:
            rp = (self.rope_parameters or {}).get(self.layer_types[l]) or {}
            if rp.get("rope_theta"):
                return float(rp["rope_theta"])
        if self.is_sliding(l):
            return self.rope_local_base_freq if self.rope_local_base_freq != 0 else 10000.0
        return self.rope_theta if self.rope_theta != 0 else 10000.0

    def validate(self) -> None:
        """config.go:229-245."""
        if self.hidden_size == 0 or self.num_hidden_layers == 0:
            raise GemmaError("gemma: config is missing hidden_size or num_hidden_layers")
        if self.head_dim % 2 != 0:
            raise GemmaError(f"gemma: head_dim {self.head_dim} must be even for RoPE")
        if self.num_key_value_heads == 0 or self.num_attention_heads % self.num_key_value_heads != 0:
            raise GemmaError(f"gemma: {self.num_attention_heads} query heads not a multiple of "
                             f"{self.num_key_value_heads} key/value heads")
        if self.hidden_activation not in ("", "gelu_pytorch_tanh"):
            raise GemmaError(f"gemma: activation {self.hidden_activation!r} not supported "
                             "(want gelu_pytorch_tanh)")
        if self.rope_scaling is not None:
            raise GemmaError("gemma: rope_scaling is set; not supported")
        if len(self.layer_types) != self.num_hidden_layers:
            raise GemmaError(f"gemma: {len(self.layer_types)} layer types for "
                             f"{self.num_hidden_layers} layers")


def _fill_variant2(c: Config) -> Config:
    """fillVariant2 (config.go:249-297): EmbeddingGemma 2's defaults and checks."""
    c.variant = 2
    if not c.layer_types:
        c.layer_types = ["full_attention" if (i + 1) % 6 == 0 else "sliding_attention"
                         for i in range(c.num_hidden_layers)]
    if c.per_layer_config is None:
        c.per_layer_config = {f"{i:02d}": {"head_dim": 512, "num_key_value_heads": 1}
                              for i, t in enumerate(c.layer_types) if t == "full_attention"}
    if c.rope_parameters is None:
        c.rope_parameters = {"sliding_attention": {"rope_theta": 10000.0, "rope_type": "default"},
                             "full_attention": {"rope_theta": 1000000.0, "rope_type": "default"}}
    for t, rp in c.rope_parameters.items():
        if rp.get("rope_type") not in (None, "", "default"):
            raise GemmaError(f"gemma: rope_type {rp.get('rope_type')!r} for {t} not supported")
    if c.embedding_dim == 0:
        c.embedding_dim = 768
    if c.hidden_size_per_layer_input == 0:
        raise GemmaError("gemma: embedding_gemma2 config without hidden_size_per_layer_input")
    c.validate()
    for l in range(c.num_hidden_layers):
        if c.head_dim_of(l) % 2 != 0:
            raise GemmaError(f"gemma: layer {l} head_dim {c.head_dim_of(l)} must be even for RoPE")
        if c.num_attention_heads % c.kv_heads_of(l) != 0:
            raise GemmaError(f"gemma: layer {l}: {c.num_attention_heads} query heads not a multiple of "
                             f"{c.kv_heads_of(l)} key/value heads")
    return c


def config_from_dict(raw: dict) -> Config:
    """LoadConfig's parsing and defaults (config.go:178-227); an
    embedding_gemma2 checkpoint's text model is read from text_config
    (config.go:174-207; its vision and audio towers are not run here)."""
    if raw.get("model_type") == "embedding_gemma2":
        c = Config()
        text = raw.get("text_config") or {}
        for f in c.__dataclass_fields__:
            if f in text and text[f] is not None and f != "variant":
                setattr(c, f, text[f])
        c.rope_scaling = text.get("rope_scaling")
        return _fill_variant2(c)
    c = Config()
    for f in c.__dataclass_fields__:
        if f in raw and raw[f] is not None:
            setattr(c, f, raw[f])
    c.rope_scaling = raw.get("rope_scaling")
    if c.sliding_window_pattern == 0:
        c.sliding_window_pattern = 6
    if not c.layer_types:
        c.layer_types = ["full_attention" if (i + 1) % c.sliding_window_pattern == 0
                         else "sliding_attention" for i in range(c.num_hidden_layers)]
    c.validate()
    return c


def LoadConfig(d) -> Config:
    """Reads config.json from a model directory (config.go:153)."""
    return config_from_dict(json.loads((Path(d) / "config.json").read_text()))


# ------------------------------------------------------------------ options
Option = Callable[["Model"], None]


def Threads(n: int) -> Option:
    """Accepted for API compatibility: the GPU path has no host thread pool."""
    return lambda m: None


def MaxTokens(n: int) -> Option:
    """Truncate inputs to at most n tokens (model.go:354-356)."""
    def f(m):
        m.max_tokens = n
    return f


def BatchTokens(n: int) -> Option:
    """Padded-token budget per forward pass (model.go:358-359)."""
    def f(m):
        m.batch_tokens = n
    return f


def WeightsBF16() -> Option:
    """Keep the bf16 projections resident as bf16 on the device and widen
    each layer's just before use (fg_model_set_weight_residency): half the
    weight bytes, identical embeddings. The reference lists this as open
    work (TODO.md: "bf16 weight storage expanded during GEMM packing")."""
    def f(m):
        m.weight_residency = _lib.WEIGHTS_BF16
    return f


@dataclass
class DenseSpec:
    w: np.ndarray          # [out, in] float32 or bf16 bits
    dtype: int
    tanh: bool = False

    @property
    def shape(self):
        return self.w.shape


_DTYPE = {"F32": _lib.DT_F32, "BF16": _lib.DT_BF16, "F16": _lib.DT_F16}


def _load_head(d: Path) -> Tuple[List[DenseSpec], bool]:
    """modules.json → Dense layers and the Normalize flag (model.go:236-310)."""
    dense, l2 = [], True
    mpath = d / "modules.json"
    if not mpath.exists():
        return dense, l2
    for mod in json.loads(mpath.read_text()):
        t = mod.get("type", "")
        if t == "sentence_transformers.sentence_transformer.modules.pooling.Pooling":
            pc = json.loads((d / mod["path"] / "config.json").read_text())
            if pc.get("pooling_mode") != "mean":
                raise GemmaError(f"gemma: pooling mode {pc.get('pooling_mode')!r} not supported, only mean")
        elif t == "sentence_transformers.models.Pooling":
            p = d / mod["path"] / "config.json"
            pc = json.loads(p.read_text()) if p.exists() else {}
            if pc.get("pooling_mode_cls_token") or pc.get("pooling_mode_lasttoken"):
                raise GemmaError("gemma: only mean pooling is supported")
        elif t == "sentence_transformers.models.Dense":
            dc = json.loads((d / mod["path"] / "config.json").read_text())
            st = read_safetensors(d / mod["path"] / "model.safetensors")
            if "linear.weight" not in st:
                raise GemmaError("gemma: Dense module without linear.weight")
            dt, w = st["linear.weight"]
            act = dc.get("activation_function", "")
            if act in ("torch.nn.modules.linear.Identity", ""):
                tanh = False
            elif act == "torch.nn.modules.activation.Tanh":
                tanh = True
            else:
                raise GemmaError(f"gemma: Dense activation {act!r} not supported")
            dense.append(DenseSpec(w, _DTYPE[dt], tanh))
        elif t in ("sentence_transformers.models.Normalize",
                   "sentence_transformers.base.modules.normalize.Normalize"):
            l2 = True
    return dense, l2


# ------------------------------------------------------------------ model
class Model:
    """A loaded encoder on one CUDA device (the reference's *gemma.Model)."""

    def __init__(self, cfg: Config, weights: Dict[str, Tuple[int, np.ndarray]],
                 dense: Sequence[DenseSpec], l2: bool = True, device: int = 0,
                 max_batch_tokens: int = 8192, options: Sequence[Option] = ()):
        self.cfg = cfg
        self.device = device
        self.max_tokens = min(cfg.max_position_embeddings or 2048, 2048)
        self.batch_tokens = 8192
        if cfg.variant == 2:
            # scores unscaled, the model card's 8192-token context (model.go:105-109)
            self.scale = 1.0
            self.max_tokens = min(cfg.max_position_embeddings or 8192, 8192)
        else:
            self.scale = 1.0 / math.sqrt(cfg.query_pre_attn_scalar)
        self.dense = list(dense)
        self.weight_residency = _lib.WEIGHTS_F32
        for o in options:
            o(self)
        lib = _lib.lib()
        L = cfg.num_hidden_layers
        self._sliding = (C.c_int * L)(*[1 if cfg.is_sliding(l) else 0 for l in range(L)])
        self._bases = (C.c_double * L)(*[cfg.rope_base(l) for l in range(L)])
        fc = _lib.Config()
        fc.hidden_size = cfg.hidden_size
        fc.intermediate_size = cfg.intermediate_size
        fc.num_layers = L
        fc.num_heads = cfg.num_attention_heads
        fc.num_kv_heads = cfg.num_key_value_heads
        fc.head_dim = cfg.head_dim
        fc.vocab_size = cfg.vocab_size
        fc.window = cfg.window() if cfg.sliding_window > 0 else 0
        fc.rms_norm_eps = float(cfg.rms_norm_eps)
        fc.attn_scale = float(np.float32(self.scale))
        fc.max_tokens = max(self.max_tokens, 1)
        fc.sliding = self._sliding
        fc.rope_base = self._bases
        if len(self.dense) > _lib.MAX_DENSE:
            raise GemmaError(f"gemma: {len(self.dense)} Dense layers (at most {_lib.MAX_DENSE})")
        fc.num_dense = len(self.dense)
        for j, d in enumerate(self.dense):
            fc.dense_out[j], fc.dense_in[j] = int(d.shape[0]), int(d.shape[1])
            fc.dense_tanh[j] = int(d.tanh)
        fc.l2_normalize = int(l2)
        if cfg.variant == 2:
            self._hd = (C.c_int * L)(*[cfg.head_dim_of(l) for l in range(L)])
            self._kv = (C.c_int * L)(*[cfg.kv_heads_of(l) for l in range(L)])
            fc.variant = 2
            fc.layer_head_dim = self._hd
            fc.layer_kv_heads = self._kv
            fc.ple_dim = cfg.hidden_size_per_layer_input
            fc.embedding_dim = cfg.embedding_dim
        h = C.c_void_p()
        _lib.check(lib.fg_model_create(C.byref(fc), device, C.byref(h)))
        self._h = h
        try:
            _lib.check(lib.fg_model_set_weight_residency(self._h, int(self.weight_residency)))
            for name, (dt, arr) in weights.items():
                self._set(name, dt, arr)
            for j, d in enumerate(self.dense):
                self._set(f"dense.{j}.linear.weight", d.dtype, d.w)
            _lib.check(lib.fg_model_finalize(self._h, int(max_batch_tokens)))
        except Exception:
            self.close()
            raise

    def _set(self, name: str, dtype: int, arr: np.ndarray) -> None:
        a = np.ascontiguousarray(arr)
        shape = (C.c_int64 * a.ndim)(*a.shape)
        _lib.check(_lib.lib().fg_model_set_weight(self._h, name.encode(), dtype, shape, a.ndim,
                                                  a.ctypes.data_as(C.c_void_p)))

    # -- the reference's accessors
    def Config(self) -> Config:
        return self.cfg

    def Dim(self) -> int:
        """Embedding width before Matryoshka truncation (model.go:336-344)."""
        if self.cfg.variant == 2:
            return self.cfg.embedding_dim
        return int(self.dense[-1].shape[0]) if self.dense else self.cfg.hidden_size

    def weight_bytes(self) -> int:
        """Device bytes held by the weights (fg_model_weight_bytes)."""
        n = _lib.lib().fg_model_weight_bytes(self._h)
        _lib.check(int(n) if n < 0 else 0)
        return int(n)

    def close(self) -> None:
        if getattr(self, "_h", None):
            _lib.lib().fg_model_destroy(self._h)
            self._h = None

    Close = close

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # -- embedBatch / Embed
    def embed_padded(self, ids: np.ndarray, lengths: np.ndarray, dim: Optional[int] = None,
                     precision: int = PREC_SPLIT, out: Optional[np.ndarray] = None) -> np.ndarray:
        """One forward over an already padded [B, T] batch (host buffers;
        pinned ones are copied without staging)."""
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        lengths = np.ascontiguousarray(lengths, dtype=np.int32)
        B, T = ids.shape
        dim = self.Dim() if dim is None else dim
        if dim < 1 or dim > self.Dim():
            raise GemmaError(f"gemma: Dim({dim}) outside 1..{self.Dim()}")
        if out is None:
            out = np.empty((B, dim), dtype=np.float32)
        elif out.shape != (B, dim) or out.dtype != np.float32 or not out.flags.c_contiguous:
            raise GemmaError("gemma: out must be a contiguous float32 [B, dim] array")
        _lib.check(_lib.lib().fg_embed_ids(self._h, ids.ctypes.data_as(C.c_void_p),
                                           lengths.ctypes.data_as(C.c_void_p), B, T, dim,
                                           precision, out.ctypes.data_as(C.c_void_p)))
        return out

    def embed_batch(self, seqs: Sequence[Sequence[int]], dim: Optional[int] = None,
                    precision: int = PREC_SPLIT) -> np.ndarray:
        """embedBatch (embed.go:118-157): right-pad with id 0, encode, pool, head."""
        B = len(seqs)
        T = max((len(s) for s in seqs), default=0)
        ids = np.zeros((B, max(T, 1)), dtype=np.int32)
        lengths = np.zeros(B, dtype=np.int32)
        for b, s in enumerate(seqs):
            ids[b, :len(s)] = s
            lengths[b] = len(s)
        return self.embed_padded(ids, lengths, dim, precision)

    def embed_device(self, d_ids, d_lengths, B: int, T: int, dim: int, d_out, stream=None,
                     precision: int = PREC_SPLIT) -> None:
        """Device-resident forward: ids/lengths/out are device pointers (ints)
        or CUDA tensors; asynchronous on `stream` (a torch stream or handle)."""
        p = lambda t: t if isinstance(t, int) else t.data_ptr()
        s = getattr(stream, "cuda_stream", stream)
        _lib.check(_lib.lib().fg_embed_ids_device(self._h, p(d_ids), p(d_lengths), B, T, dim,
                                                  precision, p(d_out), s))

    def check(self) -> None:
        """Raises if a kernel's bounded wait gave up since the last check."""
        _lib.check(_lib.lib().fg_model_check(self._h))

    def set_profiling(self, on: bool) -> None:
        """Brackets every kernel launch with CUDA events on its stream."""
        _lib.check(_lib.lib().fg_model_set_profiling(self._h, int(on)))

    def read_profile(self) -> Dict[str, dict]:
        """Per phase: device ms, launches and algorithmic work since the
        last read (FLOPs for GEMM phases, bytes for memory-bound ones)."""
        n = len(_lib.PHASES)
        ms = (C.c_double * n)()
        launches = (C.c_int64 * n)()
        work = (C.c_double * n)()
        _lib.check(_lib.lib().fg_model_read_profile(self._h, ms, launches, work, n))
        return {p: {"ms": ms[i], "launches": launches[i], "work": work[i]}
                for i, p in enumerate(_lib.PHASES)}

    def embed_ids(self, seqs: Sequence[Sequence[int]], Dim: Optional[int] = None,
                  precision: int = PREC_SPLIT) -> List[np.ndarray]:
        """(*Model).Embed (embed.go:15-80) from token ids: truncation, the
        stable length sort, greedy batches under BatchTokens and the
        overlapped host/GPU pipeline all run in fg_embed_many."""
        dim = self.Dim()
        if Dim is not None and Dim != 0:
            if Dim < 1 or Dim > dim:
                raise GemmaError(f"gemma: Dim({Dim}) outside 1..{dim}")
            dim = Dim
        n = len(seqs)
        if n == 0:
            return []
        flat, offsets = _pack(seqs)
        out = np.empty((n, dim), dtype=np.float32)
        _lib.check(_lib.lib().fg_embed_many(self._h, flat.ctypes.data_as(C.c_void_p),
                                            offsets.ctypes.data_as(C.c_void_p), n, int(self.max_tokens),
                                            int(self.batch_tokens), dim, precision,
                                            out.ctypes.data_as(C.c_void_p)))
        return list(out)


def _pack(seqs: Sequence[Sequence[int]]):
    n = len(seqs)
    lens = np.fromiter((len(s) for s in seqs), dtype=np.int64, count=n)
    offsets = np.zeros(n + 1, dtype=np.int64)
    np.cumsum(lens, out=offsets[1:])
    flat = np.zeros(max(int(offsets[-1]), 1), dtype=np.int32)
    for i, s in enumerate(seqs):
        if lens[i]:
            flat[offsets[i]:offsets[i + 1]] = s
    return flat, offsets


def embed_ids_multi(models: Sequence[Model], seqs: Sequence[Sequence[int]], Dim: Optional[int] = None,
                    precision: int = PREC_SPLIT) -> np.ndarray:
    """(*Model).Embed (embed.go:15-80) over several GPUs in one process
    (fg_embed_many_multi): the length-sorted sequences cut into one
    cost-balanced contiguous slice per model (one model per GPU, the same
    weights), each slice embedded on its own host thread, the embeddings
    returned as [len(seqs), dim] in the caller's order. BatchTokens and the
    truncation come from models[0]."""
    if not models:
        raise GemmaError("gemma: no models")
    m0 = models[0]
    dim = m0.Dim()
    if Dim is not None and Dim != 0:
        if Dim < 1 or Dim > dim:
            raise GemmaError(f"gemma: Dim({Dim}) outside 1..{dim}")
        dim = Dim
    n = len(seqs)
    out = np.empty((n, dim), dtype=np.float32)
    if n == 0:
        return out
    flat, offsets = _pack(seqs)
    hs = (C.c_void_p * len(models))(*[m._h for m in models])
    _lib.check(_lib.lib().fg_embed_many_multi(hs, len(models), flat.ctypes.data_as(C.c_void_p),
                                              offsets.ctypes.data_as(C.c_void_p), n, int(m0.max_tokens),
                                              int(m0.batch_tokens), dim, precision,
                                              out.ctypes.data_as(C.c_void_p)))
    return out


def plan_split(lengths: Sequence[int], parts: int) -> List[np.ndarray]:
    """fg_plan_split: each part's sequence indices, contiguous runs of the
    stable length order cut at equal estimated cost."""
    n = len(lengths)
    ln = np.ascontiguousarray(lengths, dtype=np.int32)
    order = np.zeros(max(n, 1), np.int32)
    bounds = np.zeros(parts + 1, np.int32)
    _lib.check(_lib.lib().fg_plan_split(ln.ctypes.data_as(C.c_void_p), n, int(parts),
                                        order.ctypes.data_as(C.c_void_p), bounds.ctypes.data_as(C.c_void_p)))
    o = order[:n].astype(np.int64)
    return [o[bounds[r]:bounds[r + 1]] for r in range(parts)]


def sequence_cost(lengths) -> np.ndarray:
    """fg_sequence_cost of each length (units: one token of a 512-token sequence)."""
    f = _lib.lib().fg_sequence_cost
    return np.array([f(int(x)) for x in np.asarray(lengths).ravel()], dtype=np.float64)


def plan_batches(lengths: Sequence[int], batch_tokens: int) -> Tuple[List[int], List[List[int]]]:
    """The batching Model.embed_ids runs (fg_plan_batches): the indices in
    stable length order and the batches as lists of indices."""
    n = len(lengths)
    ln = np.ascontiguousarray(lengths, dtype=np.int32)
    order = np.zeros(max(n, 1), np.int32)
    ends = np.zeros(max(n, 1), np.int32)
    nb = _lib.lib().fg_plan_batches(ln.ctypes.data_as(C.c_void_p), n, int(batch_tokens),
                                    order.ctypes.data_as(C.c_void_p), ends.ctypes.data_as(C.c_void_p))
    _lib.check(min(nb, 0))
    o = order[:n].tolist()
    batches, start = [], 0
    for e in ends[:nb].tolist():
        batches.append(o[start:e])
        start = e
    return o, batches


def Load(d, *options: Option, device: int = 0, max_batch_tokens: int = 8192) -> Model:
    """gemma.Load (model.go:76-232): a Hugging Face / sentence-transformers
    model directory onto CUDA device `device`."""
    d = Path(d)
    cfg = LoadConfig(d)
    files = sorted(d.glob("*.safetensors"))
    if not files:
        raise GemmaError(f"gemma: no safetensors in {d}")
    weights: Dict[str, Tuple[int, np.ndarray]] = {}
    for f in files:
        for name, (dt, arr) in read_safetensors(f).items():
            for pre in ("model.", "language_model."):
                if name.startswith(pre):
                    name = name[len(pre):]
            if dt not in _DTYPE:
                raise GemmaError(f"gemma: weight {name} has dtype {dt}")
            weights[name] = (_DTYPE[dt], arr)
    dense, l2 = _load_head(d)
    return Model(cfg, weights, dense, l2, device=device, max_batch_tokens=max_batch_tokens,
                 options=options)


def from_synthetic(cfg_dict: dict, weights_bf16: Dict[str, np.ndarray], device: int = 0,
                   max_batch_tokens: int = 8192, options: Sequence[Option] = ()) -> Model:
    """A model from in-memory weights — bf16 bits as uint16 arrays
    (ai_b200.synthetic.make_weights) or float32 arrays (make_weights_f32, an
    fp32 checkpoint) — the same path Load takes after reading the files."""
    cfg = config_from_dict(cfg_dict)

    def dt(v):
        return _lib.DT_F32 if np.asarray(v).dtype == np.float32 else _lib.DT_BF16

    body = {k: (dt(v), v) for k, v in weights_bf16.items() if not k.startswith("dense.")}
    dense = []
    j = 0
    while f"dense.{j}.linear.weight" in weights_bf16:
        v = weights_bf16[f"dense.{j}.linear.weight"]
        dense.append(DenseSpec(v, dt(v)))
        j += 1
    return Model(cfg, body, dense, True, device=device, max_batch_tokens=max_batch_tokens,
                 options=options)
