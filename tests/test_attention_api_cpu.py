"""Host-side surface of the drop-in ``attention_exact`` module (no GPU):
the additive causal mask and the argument errors raised before any kernel."""

import numpy as np
import pytest
import torch

from oracle.segmented_attention import build_causal_mask as oracle_mask
from rfsn_b200 import attention_exact


@pytest.mark.parametrize("q_len,k_len,q_start,k_start", [
    (1, 1, 0, 0),
    (1, 4096, 8191, 4096),      # decode token after the keys
    (7, 13, 20, 10),            # causal diagonal inside the key range
    (5, 9, 0, 3),               # keys after every query: all masked
    (64, 64, 128, 128),         # prefill chunk against itself
    (3, 0, 5, 0),               # no keys
])
def test_causal_mask_matches_reference_formula(q_len, k_len, q_start, k_start):
    got = attention_exact.build_causal_mask(q_len, k_len, q_start, k_start)
    want = oracle_mask(q_len, k_len, q_start, k_start)
    assert got.dtype == torch.float32 and tuple(got.shape) == (1, 1, q_len, k_len)
    assert np.array_equal(got.numpy(), want)
    if k_len:
        assert set(np.unique(want).tolist()) <= {0.0, np.float32(-1e9)}


def test_empty_segment_list_raises_like_reference():
    # attention_exact.py:133-134
    with pytest.raises(RuntimeError, match="requires at least one KV segment"):
        attention_exact.run_segmented_attention(torch.zeros(1, 2, 1, 4), [], 0)
