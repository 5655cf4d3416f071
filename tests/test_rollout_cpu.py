"""Rollout helpers on CPU: the 2 bpp unpack/pack and the config-5 policy shape."""

from __future__ import annotations

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from gbxcule_b200 import rollout  # noqa: E402


def test_unpack_matches_bit_layout_and_roundtrips():
    rng = np.random.default_rng(3)
    packed = torch.as_tensor(rng.integers(0, 256, (5, 72, 20), dtype=np.uint8))
    px = rollout.unpack_2bpp_u8(packed)
    assert px.shape == (5, 72, 80) and px.dtype == torch.uint8
    p = packed.numpy().astype(np.int32)
    want = np.stack([(p >> s) & 3 for s in (0, 2, 4, 6)], axis=-1).reshape(5, 72, 80)
    assert np.array_equal(px.numpy(), want)
    assert torch.equal(rollout.pack_2bpp_u8(px), packed)
    with pytest.raises(ValueError):
        rollout.unpack_2bpp_u8(packed.to(torch.int32))


def test_policy_shape():
    pol = rollout.make_policy("cpu", dtype=torch.float32)
    logits = pol(torch.randint(0, 4, (3, 72, 80), dtype=torch.uint8))
    assert logits.shape == (3, 9)
