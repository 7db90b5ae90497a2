"""EmbeddingGemma 2's configuration on the host (no GPU): the nested
text_config, the per-layer geometry and rotary bases, the window bound and
the checks of fillVariant2 (models/gemma/config.go:249-362), mirroring the
reference's TestConfig2 (gemma2_test.go)."""
import pytest

from ai_b200 import gemma
from ai_b200 import synthetic as S


def test_config2_geometry_and_bases():
    raw = {"model_type": "embedding_gemma2", "vision_config": {"hidden_size": 768},
           "text_config": dict(S.EMBEDDINGGEMMA2_TEXT)}
    raw["text_config"]["max_position_embeddings"] = 262144
    c = gemma.config_from_dict(raw)
    assert c.variant == 2 and c.hidden_size == 512 and c.embedding_dim == 768
    for layer, hd, kv, sliding, base in [(0, 256, 2, True, 1e4), (4, 256, 2, True, 1e4),
                                         (5, 512, 1, False, 1e6), (11, 512, 1, False, 1e6)]:
        assert c.head_dim_of(layer) == hd
        assert c.kv_heads_of(layer) == kv
        assert c.is_sliding(layer) == sliding
        assert c.rope_base(layer) == base
    assert c.window() == 513  # an inclusive radius of 512


def test_config2_defaults():
    t = {k: v for k, v in S.EMBEDDINGGEMMA2_TEXT.items()
         if k not in ("per_layer_config", "rope_parameters", "embedding_dim")}
    c = gemma.config_from_dict({"model_type": "embedding_gemma2", "text_config": t})
    assert c.layer_types[5] == "full_attention" and c.layer_types[4] == "sliding_attention"
    assert c.head_dim_of(5) == 512 and c.kv_heads_of(5) == 1 and c.head_dim_of(0) == 256
    assert c.rope_base(0) == 1e4 and c.rope_base(11) == 1e6
    assert c.embedding_dim == 768


def test_config2_rejections():
    t = dict(S.EMBEDDINGGEMMA2_TEXT)
    t.pop("hidden_size_per_layer_input")
    with pytest.raises(gemma.GemmaError, match="hidden_size_per_layer_input"):
        gemma.config_from_dict({"model_type": "embedding_gemma2", "text_config": t})
    t = dict(S.EMBEDDINGGEMMA2_TEXT)
    t["rope_parameters"] = {"full_attention": {"rope_theta": 1e6, "rope_type": "yarn"}}
    with pytest.raises(gemma.GemmaError, match="rope_type"):
        gemma.config_from_dict({"model_type": "embedding_gemma2", "text_config": t})
    t = dict(S.EMBEDDINGGEMMA2_TEXT)
    t["per_layer_config"] = {"05": {"head_dim": 512, "num_key_value_heads": 3}}
    with pytest.raises(gemma.GemmaError, match="key/value heads"):
        gemma.config_from_dict({"model_type": "embedding_gemma2", "text_config": t})


def test_oracle_batch_invariance_and_unit_norm():
    import numpy as np

    from oracle import gemma2 as G

    cfg = S.eg2_small_config()
    w = S.make_weights_eg2(cfg, seed=1)
    o = G.from_bf16(cfg, w)
    ids = S.make_ids(3, 80, 2, 4096)
    lengths = np.array([80, 37, 1])
    e = o.embed_padded(ids, lengths)
    assert np.allclose(np.linalg.norm(e, axis=1), 1.0)
    for b in range(3):
        alone = o.embed_padded(ids[b:b + 1, :lengths[b]], lengths[b:b + 1])
        assert np.abs(alone[0] - e[b]).max() < 1e-12
