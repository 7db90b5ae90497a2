"""CPU tests of the host side: the C ABI library loads and exports every
symbol include/fgemma.h declares (no device calls), config parsing and the
derived window / layer types / RoPE bases (config.go:153-245, 325-362),
Embed's length sort and greedy batching (embed.go:15-80), and argument
checking that needs no GPU."""
import ctypes as C
import json
import re
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent


def _declared():
    text = (ROOT / "include" / "fgemma.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(fg_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    from ai_b200 import _lib

    lib = _lib.lib()
    names = _declared()
    assert len(names) >= 15
    for n in names:
        assert hasattr(lib, n), n
    assert set(names) <= set(_lib.SIGNATURES), set(names) - set(_lib.SIGNATURES)


def test_device_count_without_gpu_is_zero_or_more():
    from ai_b200 import _lib

    assert _lib.lib().fg_device_count() >= 0


def test_model_create_without_device_fails_cleanly():
    import torch

    from ai_b200 import _lib

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    cfg = _lib.Config()
    L = 1
    sl = (C.c_int * L)(1)
    rb = (C.c_double * L)(1e4)
    cfg.hidden_size, cfg.intermediate_size, cfg.num_layers = 768, 1152, L
    cfg.num_heads, cfg.num_kv_heads, cfg.head_dim, cfg.vocab_size = 3, 1, 256, 10
    cfg.max_tokens, cfg.sliding, cfg.rope_base = 16, sl, rb
    h = C.c_void_p()
    rc = _lib.lib().fg_model_create(C.byref(cfg), 0, C.byref(h))
    assert rc == _lib.FG_ENODEV
    assert b"device" in _lib.lib().fg_last_error()


def test_config_defaults_and_derivations():
    from ai_b200 import gemma, synthetic as S

    c = gemma.config_from_dict(dict(S.EMBEDDINGGEMMA_300M))
    assert c.window() == 257  # 512/2 + 1 for bidirectional models
    assert [l for l in range(24) if not c.is_sliding(l)] == [5, 11, 17, 23]
    assert c.rope_base(0) == 1e4 and c.rope_base(5) == 1e6
    causal = dict(S.EMBEDDINGGEMMA_300M, use_bidirectional_attention=False)
    assert gemma.config_from_dict(causal).window() == 512
    with pytest.raises(gemma.GemmaError):
        gemma.config_from_dict(dict(S.EMBEDDINGGEMMA_300M, head_dim=255))
    with pytest.raises(gemma.GemmaError):
        gemma.config_from_dict(dict(S.EMBEDDINGGEMMA_300M, hidden_activation="relu"))
    with pytest.raises(gemma.GemmaError):
        gemma.config_from_dict(dict(S.EMBEDDINGGEMMA_300M, layer_types=["full_attention"]))


def test_load_config_and_head_from_a_model_dir(tmp_path):
    from ai_b200 import gemma, synthetic as S

    cfg = S.small_config(layers=1, vocab=64)
    w = S.make_weights(cfg, seed=0)
    S.write_model_dir(tmp_path, cfg, w)
    c = gemma.LoadConfig(tmp_path)
    assert c.num_hidden_layers == 1 and c.vocab_size == 64
    dense, l2 = gemma._load_head(tmp_path)
    assert [d.shape for d in dense] == [(3072, 768), (768, 3072)] and l2
    st = S.read_safetensors(tmp_path / "model.safetensors")
    assert st["embed_tokens.weight"][0] == "BF16"
    assert np.array_equal(st["embed_tokens.weight"][1], w["embed_tokens.weight"])


def test_embed_batches_by_length_under_the_token_budget():
    """fg_embed_many's batching (embed.go:46-74), on the host only."""
    from ai_b200 import gemma

    lengths = [5, 3, 9, 3, 1, 7]
    order, batches = gemma.plan_batches(lengths, 12)
    # stable ascending order: 1, 3, 3, 5, 7, 9; maxLen·(n+1) ≤ 12
    assert order == [4, 1, 3, 0, 5, 2]
    assert [[lengths[i] for i in b] for b in batches] == [[1, 3, 3], [5], [7], [9]]
    # a sequence longer than the budget runs alone; empty input, zero lengths
    assert gemma.plan_batches([20, 2, 2], 8)[1] == [[1, 2], [0]]
    assert gemma.plan_batches([], 8) == ([], [])
    assert gemma.plan_batches([0, 0, 0], 2)[1] == [[0, 1, 2]]
    rng = np.random.default_rng(3)
    ln = rng.integers(0, 600, 500).tolist()
    order, batches = gemma.plan_batches(ln, 4096)
    assert sorted(order) == list(range(500))
    assert [ln[i] for i in order] == sorted(ln)
    assert sum(batches, []) == order
    for b in batches:
        assert len(b) == 1 or max(ln[i] for i in b) * len(b) <= 4096


def test_tensor_ops_reject_bad_shapes_before_any_device_call():
    import torch

    from ai_b200 import tensor as T

    x = torch.zeros(3, 4)
    with pytest.raises(T.TensorError):
        T.MatMul(x, torch.zeros(5, 2))  # not CUDA and mismatched
