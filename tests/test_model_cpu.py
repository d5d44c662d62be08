"""Model driver host logic (no GPU): parameter names/shapes against the
reference's own parameter tree (the golden tiny model's weights were taken
from ``tree_flatten(RFSNMLX.parameters())``), weight loading errors, and the
prefill/decode bounds checks of model.py:74-104."""

import numpy as np
import pytest
import torch

from _util import GOLDEN
from rfsn_b200.config import RFSNConfig, RuntimeMode
from rfsn_b200.model import RFSNModel


def tiny_config(tmp_path, **kw):
    args = dict(hidden_dim=128, num_heads=2, num_kv_heads=2, head_dim=64, num_layers=1, vocab_size=128,
                hot_capacity=8, block_size_seq=4, rope_base=10000.0, ffn_multiplier=4, model_dtype="float32",
                runtime_mode=RuntimeMode.ARCHIVED, disk_cache_dir=str(tmp_path), session_id="tiny")
    args.update(kw)
    return RFSNConfig(**args)


class _FakeLayer:
    def __init__(self, hot_end):
        self.hot_end = hot_end


class _FakeCache:
    def __init__(self, hot_end):
        self._l = _FakeLayer(hot_end)

    def layer(self, i):
        return self._l


def test_parameter_names_and_shapes_match_reference_tree(tmp_path):
    g = np.load(GOLDEN / "tiny_model_golden.npz")
    ref = {k[2:]: g[k].shape for k in g.files if k.startswith("w/")}
    model = RFSNModel(tiny_config(tmp_path), device="cpu")
    shapes = model.parameter_shapes()
    # the golden stores every non-norm parameter; norms keep their init (ones / zeros)
    assert set(ref) == {k for k in shapes if "norm" not in k}
    for k, s in ref.items():
        assert shapes[k] == tuple(s), k
    model.load_weights({k: g["w/" + k] for k in ref})
    np.testing.assert_array_equal(model.params["layers.0.q_proj.weight"].numpy(), g["w/layers.0.q_proj.weight"])
    assert torch.all(model.params["layers.0.attn_norm.weight"] == 1)
    assert torch.all(model.params["norm.bias"] == 0)


def test_load_weights_rejects_unknown_and_misshaped(tmp_path):
    model = RFSNModel(tiny_config(tmp_path), device="cpu")
    with pytest.raises(ValueError, match="not in model"):
        model.load_weights({"layers.0.bogus.weight": np.zeros((2, 2), np.float32)})
    with pytest.raises(ValueError, match="Expected shape"):
        model.load_weights({"embed_tokens.weight": np.zeros((2, 2), np.float32)})
    with pytest.raises(ValueError, match="Missing parameters"):
        model.load_weights({"embed_tokens.weight": np.zeros((128, 128), np.float32)}, strict=True)


def test_bounds_checks_match_reference_messages(tmp_path):
    model = RFSNModel(tiny_config(tmp_path, max_position_embeddings=16), device="cpu")
    with pytest.raises(ValueError, match="max_position_embeddings=16"):
        model._validate_prefill_bounds(_FakeCache(10), 7)
    assert model._validate_prefill_bounds(_FakeCache(10), 6) == 10
    with pytest.raises(ValueError, match="decode_step expected pos=5 from cache state, got pos=4"):
        model._validate_decode_bounds(_FakeCache(5), 4)
    with pytest.raises(ValueError, match="Decode would exceed"):
        model._validate_decode_bounds(_FakeCache(16), 16)
    exact = RFSNModel(tiny_config(tmp_path, runtime_mode=RuntimeMode.EXACT), device="cpu")
    with pytest.raises(RuntimeError, match="hot-window only"):
        exact._validate_prefill_bounds(_FakeCache(4), 5)
    with pytest.raises(RuntimeError, match="hot-window only"):
        exact._validate_decode_bounds(_FakeCache(8), 8)
    with pytest.raises(ValueError, match="at least one token"):
        model.prefill(np.zeros((1, 0), np.int32), _FakeCache(0))


def test_greedy_and_sampling_rules():
    logits = torch.tensor([[0.1, 2.0, -1.0, 0.5]])
    assert int(RFSNModel._sample(logits, 0.0, 1.0, 0, 1.0, torch.zeros((1, 1), dtype=torch.long))[0]) == 1
    gen = torch.Generator().manual_seed(0)
    # top-k 1 leaves only the argmax
    for _ in range(5):
        t = RFSNModel._sample(logits, 1.0, 1.0, 1, 1.0, torch.zeros((1, 1), dtype=torch.long), gen)
        assert int(t[0]) == 1
    # a repetition penalty on the argmax (positive logit divided) can move the choice under top-k 1
    t = RFSNModel._sample(logits, 1.0, 1.0, 1, 100.0, torch.tensor([[1]]), gen)
    assert int(t[0]) == 3


def test_standalone_layer_has_the_reference_surface(tmp_path):
    """RFSNLayerMLX(config, layer_idx) builds a layer with its own parameters;
    q/k/v and gate/up are row views of its fused matrices, exposed through the
    reference's ``.weight`` attributes."""
    import torch

    from rfsn_b200 import RFSNLayerMLX

    cfg = tiny_config(tmp_path)
    layer = RFSNLayerMLX(cfg, 0, device="cpu")
    H, Hkv, D, Hd, Fd = cfg.num_heads, cfg.num_kv_heads, cfg.head_dim, cfg.hidden_dim, cfg.ffn_dim
    assert tuple(layer.q_proj.weight.shape) == (H * D, Hd)
    assert tuple(layer.k_proj.weight.shape) == (Hkv * D, Hd)
    assert tuple(layer.down_proj.weight.shape) == (Hd, Fd)
    assert torch.equal(layer.attn_norm.weight, torch.ones(Hd, dtype=layer.attn_norm.weight.dtype))
    from rfsn_b200.layer import RFSNLayerMLX as from_layer_module, RFSNLayerNorm

    assert from_layer_module is RFSNLayerMLX and isinstance(layer.ffn_norm, RFSNLayerNorm)
    layer.k_proj.weight.fill_(0.5)  # a write through the reference attribute lands in the fused matrix
    assert bool((layer.w_qkv[H * D:(H + Hkv) * D] == 0.5).all())
    assert layer.up_proj.weight.data_ptr() == layer.w_gate_up[Fd:].data_ptr()
