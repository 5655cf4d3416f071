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


def test_space_to_depth_conv_computes_the_stride_two_conv():
    """Conv(1->32, k4, s2) over the frame equals the k2 stride-1 convolution
    of its 2x2 space-to-depth with the rearranged weight (fp32, CPU)."""
    import torch
    import torch.nn.functional as F

    from gbxcule_b200 import rollout

    g = torch.Generator().manual_seed(7)
    x = torch.randint(0, 4, (3, 1, 72, 80), generator=g).float() / 3.0
    w = torch.randn(32, 1, 4, 4, generator=g)
    b = torch.randn(32, generator=g)
    want = F.conv2d(x, w, b, stride=2)
    s = rollout.s2d_frames(x)
    assert s.shape == (3, 36, 40, 4)
    assert torch.equal(s[:, 5, 7, 3], x[:, 0, 11, 15]) and torch.equal(s[:, 5, 7, 2], x[:, 0, 11, 14])
    got = F.conv2d(s.permute(0, 3, 1, 2), rollout.s2d_weight(w), b, stride=1)
    assert got.shape == want.shape == (3, 32, 35, 39)
    assert torch.allclose(got, want, atol=1e-5)


def test_s2d_weight_cache_follows_in_place_updates():
    """The space-to-depth weight the policy caches is rebuilt after an in-place
    update of the first convolution's weight (an optimizer step)."""
    import torch

    from gbxcule_b200 import rollout

    pol = rollout.make_policy("cpu", dtype=torch.float32)
    c1 = pol.conv[0]
    key0 = (c1.weight.data_ptr(), c1.weight._version, c1.weight.dtype)  # the cache key of _cached
    with torch.no_grad():
        c1.weight.mul_(2.0)
    assert (c1.weight.data_ptr(), c1.weight._version, c1.weight.dtype) != key0


def test_nhwc_head_equals_the_module_head():
    """The policy head read in NHWC feature order with the permuted first-layer
    weight computes the module's NCHW-flatten head (fp32, CPU)."""
    import torch

    from gbxcule_b200 import rollout

    pol = rollout.make_policy("cpu", dtype=torch.float32)
    g = torch.Generator().manual_seed(9)
    x = torch.randn(4, 64, 15, 17, generator=g).contiguous(memory_format=torch.channels_last)
    with torch.no_grad():
        want = pol.head(x.flatten(1))
        got = pol._head_nhwc(x)
    assert torch.allclose(got, want, atol=1e-5, rtol=1e-5)
