"""RoPE of a layer called with explicit tables, or without them in a 16-bit
model (layer.py:118-135): the table-driven RoPE/append kernel against the
reference's own outputs (tests/golden/rope_golden.npz, written by the
reference's build_rope_tables / _apply_rope) and, through the cache and the
layer, against the oracle."""

import ctypes
import tempfile

import numpy as np
import pytest
import torch

from _util import GOLDEN, to_device_storage
from oracle.numerics import from_storage, round_to_dtype
from oracle.rope import apply_rope_in, promoted_dtype, rope_tables_in
from oracle.segmented_attention import run_segmented_attention

pytestmark = pytest.mark.gpu
ATOL = 2e-3
TORCH = {"bfloat16": torch.bfloat16, "float16": torch.float16, "float32": torch.float32}


def _golden_cases():
    data = np.load(GOLDEN / "rope_golden.npz")
    return data, [str(n) for n in data["__cases__"]]


@pytest.mark.parametrize("name", _golden_cases()[1])
def test_table_rope_append_equals_the_reference_bit_for_bit(name):
    """Given the reference's tables, the rotated q (float32 holding the promoted
    dtype's values) and the ring's k (rounded to the cache dtype) equal the
    reference's _apply_rope output exactly; v is appended unchanged."""
    from rfsn_b200 import _native as native

    data, _ = _golden_cases()
    xd, td, od = (str(x) for x in data[f"{name}/dtypes"])
    H, L, D, start = (int(x) for x in data[f"{name}/meta"])
    assert od == promoted_dtype(xd, td)
    x = to_device_storage(data[f"{name}/x"], xd).reshape(1, H, L, D)
    cos_t = to_device_storage(data[f"{name}/cos"], td).reshape(L, D)
    sin_t = to_device_storage(data[f"{name}/sin"], td).reshape(L, D)
    want = data[f"{name}/out"]
    cap = 8
    k_arena = torch.zeros((H, cap, D), dtype=TORCH[xd], device="cuda")
    v_arena = torch.zeros_like(k_arena)
    arena = native.Arena(k_arena, v_arena)
    v = (x * 0.5 + 1.0).contiguous()
    q_out = torch.empty((1, H, L, D), dtype=torch.float32, device="cuda")
    inv = torch.zeros(D // 2, dtype=torch.float32, device="cuda")
    native.check(native.lib().rfsn_rope_append_tables(
        x.data_ptr(), x.data_ptr(), v.data_ptr(), native.dtype_code(x.dtype), cos_t.data_ptr(), sin_t.data_ptr(),
        native.dtype_code(cos_t.dtype), inv.data_ptr(), start, 1, H, H, L, D, q_out.data_ptr(), arena.handle, 0, cap,
        cap - 2, native.stream_ptr()), "rfsn_rope_append_tables")
    torch.cuda.synchronize()
    np.testing.assert_array_equal(q_out.cpu().numpy(), want)
    slots = [(cap - 2 + l) % cap for l in range(L)]  # the write wraps around the ring
    k_ring = k_arena[:, slots].float().cpu().numpy()[None]
    np.testing.assert_array_equal(k_ring, round_to_dtype(want, xd))
    np.testing.assert_array_equal(v_arena[:, slots].float().cpu().numpy()[None], v.float().cpu().numpy())
    arena.close()


def _cfg(dtype, H, Hkv, D, cap, bs, tmp, base):
    from rfsn_b200 import RFSNConfig

    return RFSNConfig(hidden_dim=H * D, num_heads=H, num_kv_heads=Hkv, head_dim=D, num_layers=1, hot_capacity=cap,
                      warm_capacity=1 << 20, cold_capacity=1 << 21, block_size_seq=bs, model_dtype=dtype,
                      rope_base=base, disk_cache_dir=tmp)


@pytest.mark.parametrize("dtype", ["bfloat16", "float16"])
def test_attention_step_with_model_dtype_tables_matches_oracle(dtype):
    """Without tables a 16-bit layer rotates q and k with tables built in the
    model dtype and 16-bit arithmetic (not the float32 rotation of the model's
    own flow): a prefill chunk and decode steps across seals, the ring's k and
    the attention output checked against the oracle's restatement."""
    from rfsn_b200 import LayerKVCache
    from rfsn_b200.layer import attention_step_tables

    H, Hkv, D, cap, bs, base = 16, 4, 128, 64, 16, 500000.0
    chunks = [40, 1, 1, 1, 30, 1]
    total = sum(chunks)
    rng = np.random.default_rng(41)
    q = rng.standard_normal((1, H, total, D)).astype(np.float32)
    k = rng.standard_normal((1, Hkv, total, D)).astype(np.float32)
    v = rng.standard_normal((1, Hkv, total, D)).astype(np.float32)
    tdt = TORCH[dtype]
    r = lambda x: round_to_dtype(x, dtype)  # noqa: E731
    cos_t, sin_t = rope_tables_in(D, base, total, 0, dtype)
    k_rot = apply_rope_in(r(k), cos_t, sin_t, dtype)
    ulp = {"bfloat16": 2.0 ** -7, "float16": 2.0 ** -10}[dtype]
    with tempfile.TemporaryDirectory() as tmp:
        c = LayerKVCache(_cfg(dtype, H, Hkv, D, cap, bs, tmp, base), 1, H, Hkv, session_id="t")
        pos = 0
        for n in chunks:
            sl = slice(pos, pos + n)
            out = attention_step_tables(torch.from_numpy(q[:, :, sl]).to(tdt).cuda(),
                                        torch.from_numpy(k[:, :, sl]).to(tdt).cuda(),
                                        torch.from_numpy(v[:, :, sl]).to(tdt).cuda(), c, pos).cpu().numpy()
            q_rot = apply_rope_in(r(q[:, :, sl]), cos_t[sl], sin_t[sl], dtype)
            ref = run_segmented_attention(q_rot, [(k_rot[:, :, :pos + n], r(v[:, :, :pos + n]), 0)], pos, grouped=True)
            assert float(np.abs(out - ref).max()) <= ATOL
            # the newest keys in the ring: almost all equal; the float32 cos/sin of the
            # table build (CUDA vs numpy, both within an ulp) can flip a table entry's
            # 16-bit rounding, which moves the products and the sum by an ulp or two
            hot = list(c.get_hot_attention_segments())
            k_dev = torch.cat([s[0] for s in hot], dim=2)[:, :, -n:].float().cpu().numpy()
            diff = np.abs(k_dev - k_rot[:, :, sl])
            assert float(np.mean(diff > 0)) <= 0.03, float(np.mean(diff > 0))
            assert np.all(diff <= 4 * ulp * np.maximum(np.abs(k_rot[:, :, sl]), 1.0))
            pos += n
        assert c.get_block_stats()["total_blocks"] > 0


def test_standalone_bf16_layer_honours_rope_tables(tmp_path):
    """RFSNLayerMLX in bf16 with the reference's positional call (x, cache,
    rope_tables, start_pos): None builds bf16 tables, so it equals a call
    with those tables passed in; float32 tables passed in give the model's
    own float32 rotation; and the two flows differ."""
    from rfsn_b200 import RFSNCache, RFSNLayerMLX
    from rfsn_b200.model import MODEL_ROPE_TABLES

    H, Hkv, D, base = 8, 2, 128, 500000.0

    def cfg(sub):
        from rfsn_b200 import RFSNConfig

        return RFSNConfig(hidden_dim=H * D, num_heads=H, num_kv_heads=Hkv, head_dim=D, num_layers=1,
                          vocab_size=128, hot_capacity=32, warm_capacity=4096, cold_capacity=8192, block_size_seq=8,
                          model_dtype="bfloat16", rope_base=base, disk_cache_dir=str(tmp_path / sub))

    layer = RFSNLayerMLX(cfg("w"), 0, device="cuda")
    owners = {m: RFSNCache(cfg(m), batch_size=1, device="cuda") for m in ("none", "bf16", "f32", "model")}
    caches = {m: c.layer(0) for m, c in owners.items()}
    gen = torch.Generator(device="cuda").manual_seed(7)
    pos = 0
    for L in (20, 1, 1, 12):  # seals of the 32-token ring along the way
        x = (torch.randn((1, L, H * D), generator=gen, device="cuda")).to(torch.bfloat16)
        c32, s32 = rope_tables_in(D, base, L, pos, "float32")
        c16, s16 = rope_tables_in(D, base, L, pos, "bfloat16")
        t32 = (torch.from_numpy(c32).cuda(), torch.from_numpy(s32).cuda())
        t16 = (torch.from_numpy(c16).to(torch.bfloat16).cuda(), torch.from_numpy(s16).to(torch.bfloat16).cuda())
        out = {
            "none": layer(x, caches["none"], None, pos),
            "bf16": layer(x, caches["bf16"], t16, pos),
            "f32": layer(x, caches["f32"], t32, pos),
            "model": layer(x, caches["model"], MODEL_ROPE_TABLES, pos),
        }
        tol = 2.0 ** -6 * float(out["none"].float().abs().max())  # a bf16 ulp or two of the output scale
        assert float((out["none"].float() - out["bf16"].float()).abs().max()) <= tol
        assert float((out["f32"].float() - out["model"].float()).abs().max()) <= tol
        pos += L
    # 16-bit and float32 rotations do give different keys
    k16 = torch.cat([s[0] for s in caches["none"].get_attention_segments()], dim=2).float()
    k32 = torch.cat([s[0] for s in caches["model"].get_attention_segments()], dim=2).float()
    assert not torch.equal(k16, k32)
