"""Pins the oracle to the reference: the golden fixtures were produced by the
reference's own modules (tests/golden/make_golden.py)."""

import numpy as np
import pytest

from _util import GOLDEN as GOLDEN_DIR
from _util import golden_attention_cases, load_json
from oracle.kv_ring import RingOracle
from oracle.numerics import bf16_bits_to_f32, f32_to_bf16_bits, from_storage
from oracle.segmented_attention import merge_partials, run_segmented_attention

CASES = golden_attention_cases()


@pytest.mark.parametrize("case", CASES, ids=[c["name"] for c in CASES])
@pytest.mark.parametrize("grouped", [False, True])
def test_oracle_attention_matches_reference(case, grouped):
    segs = [(from_storage(k, case["dtype"]), from_storage(v, case["dtype"]), s) for k, v, s in case["segs"]]
    out = run_segmented_attention(case["q"], segs, case["q_start"], grouped=grouped)
    np.testing.assert_allclose(out, case["out"], atol=2e-6, rtol=0)


def test_oracle_empty_segments_raise_like_reference():
    with pytest.raises(RuntimeError, match="at least one KV segment"):
        run_segmented_attention(np.zeros((1, 1, 1, 4), np.float32), [], 0)


def test_oracle_lse_merge_equals_unsplit():
    case = CASES[1]
    segs = [(from_storage(k, case["dtype"]), from_storage(v, case["dtype"]), s) for k, v, s in case["segs"]]
    full, _ = run_segmented_attention(case["q"], segs, case["q_start"], return_lse=True)
    parts = [run_segmented_attention(case["q"], segs[i:i + 2], case["q_start"], return_lse=True) for i in (0, 2, 4)]
    merged = merge_partials([p[0] for p in parts], [p[1] for p in parts])
    np.testing.assert_allclose(merged, full, atol=2e-6)


@pytest.mark.parametrize("case", CASES[:4], ids=[c["name"] for c in CASES[:4]])
def test_oracle_rows_at_explicit_positions_equal_the_contiguous_chunk(case):
    """Sampled query rows given with their own positions reproduce the same rows
    of the contiguous evaluation (used to check long prefill chunks by sample)."""
    segs = [(from_storage(k, case["dtype"]), from_storage(v, case["dtype"]), s) for k, v, s in case["segs"]]
    q = case["q"]
    Lq = q.shape[2]
    full, full_lse = run_segmented_attention(q, segs, case["q_start"], return_lse=True)
    rows = sorted({0, Lq - 1, Lq // 2})
    part, part_lse = run_segmented_attention(q[:, :, rows], segs, case["q_start"], return_lse=True,
                                             q_positions=[case["q_start"] + r for r in rows])
    np.testing.assert_allclose(part, full[:, :, rows], atol=2e-6, rtol=0)
    np.testing.assert_allclose(part_lse, full_lse[:, :, rows], atol=2e-6, rtol=1e-6)


ROPE = np.load(GOLDEN_DIR / "rope_golden.npz")


@pytest.mark.parametrize("name", [str(n) for n in ROPE["__cases__"]])
def test_oracle_rope_in_table_dtype_matches_reference(name):
    """The rotation with tables in the model dtype or another dtype, every op
    rounded to the promoted dtype, equals the reference's _apply_rope bit for
    bit; the tables agree to the float32 trig and inv_freq ulps (scaled by the
    position, since inv_freq's last bit moves the angle by position x ulp)."""
    from oracle.rope import apply_rope_in, promoted_dtype, rope_tables_in

    xd, td, _ = (str(x) for x in ROPE[f"{name}/dtypes"])
    H, L, D, start = (int(x) for x in ROPE[f"{name}/meta"])
    x = from_storage(ROPE[f"{name}/x"], xd)
    c = from_storage(ROPE[f"{name}/cos"], td)
    s = from_storage(ROPE[f"{name}/sin"], td)
    np.testing.assert_array_equal(apply_rope_in(x, c, s, promoted_dtype(xd, td)), ROPE[f"{name}/out"])
    c2, s2 = rope_tables_in(D, float(ROPE[f"{name}/base"]), L, start, td)
    bound = (start + L) * 2.0 ** -23 * 2 + {"float32": 0.0, "bfloat16": 2.0 ** -8, "float16": 2.0 ** -11}[td]
    assert np.abs(c2 - c).max() <= bound and np.abs(s2 - s).max() <= bound


RING = load_json("ring_traces.json")


@pytest.mark.parametrize("name", sorted(RING))
def test_ring_oracle_matches_reference_trace(name):
    sc = RING[name]
    ring = RingOracle(sc["hot_capacity"], sc["block_size"], exact_mode=sc["mode"] == "exact")
    for step in sc["steps"]:
        n = step["incoming"]
        if "error" in step:
            with pytest.raises(RuntimeError) as err:
                ring.evict_for_append(n)
                ring.append(n)
            assert str(err.value) == step["error"]
            continue
        ring.evict_for_append(n)
        ring.append(n)
        assert (ring.head, ring.length, ring.start) == (step["hot_head_index"], step["hot_seq_len"], step["hot_start"])
        assert ring.write_index == step["hot_write_index"]
        assert ring.end == step["hot_end"]
        assert [list(s) for s in ring.sealed] == [[b["start"], b["end"]] for b in step["blocks"]]
        hot = [[s, n_] for _, n_, s in ring.hot_spans()]
        assert [[b["start"], b["end"] - b["start"]] for b in step["blocks"]] + hot == step["segments"]


def test_bf16_rounding_is_round_to_nearest_even():
    x = np.array([1.0, 1.00390625, 1.01171875, -3.0e-3, 65504.0, 1e-30], np.float32)
    y = bf16_bits_to_f32(f32_to_bf16_bits(x))
    import torch

    ref = torch.from_numpy(x).to(torch.bfloat16).to(torch.float32).numpy()
    np.testing.assert_array_equal(y, ref)
