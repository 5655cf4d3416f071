"""Policy rollouts on packed observations (the reference's RL loop shape).

The reference's RL loops (``src/gbxcule/rl/``) render packed 2 bpp frames,
unpack them with a 256 x 4 lookup table (``rl/packed_pixels.py:26-71``), run
a torch policy on them, sample one action per env and call ``step_torch``;
finished episodes are restored from a ``ResetCache``. This module is that
loop over ``GbxVecCudaBackend``: frames go from libgbx's packed buffer to the
policy without leaving the GPU, and every tensor stays on the backend's
device and current stream.

``PixelPolicy`` is the config-5 benchmark network: bf16
Conv(1->32, k4, s2) -> Conv(32->64, k3, s2) -> Conv(64->64, k3, s1) ->
Linear(., 512) -> Linear(512, 9) with ReLUs, on frames scaled by 1/3 (the
strides are not given by the benchmark; 2/2/1 are used).
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any, Callable

_LUT: dict[str, Any] = {}


def unpack_lut(device) -> Any:
    """[256, 4] uint8: byte -> its four 2-bit pixels, first pixel in bits 0-1."""
    import torch

    key = str(device)
    if key not in _LUT:
        v = torch.arange(256, dtype=torch.int32)
        _LUT[key] = torch.stack([(v >> s) & 3 for s in (0, 2, 4, 6)], dim=1).to(torch.uint8).to(device)
    return _LUT[key]


_SHIFTS: dict[str, Any] = {}


def unpack_2bpp_u8(packed) -> Any:
    """Unpack uint8 2 bpp bytes along the last axis (rl/packed_pixels.py:62-71).

    Same result as the 256 x 4 lookup table (first pixel in bits 0-1),
    computed as one broadcast shift-and-mask on uint8, without an int64
    index tensor.
    """
    import torch

    if packed.dtype is not torch.uint8:
        raise ValueError("packed_u8 must be uint8")
    key = str(packed.device)
    if key not in _SHIFTS:
        _SHIFTS[key] = torch.tensor([0, 2, 4, 6], dtype=torch.uint8, device=packed.device)
    out = torch.bitwise_right_shift(packed.unsqueeze(-1), _SHIFTS[key]).bitwise_and_(3)
    return out.reshape(*packed.shape[:-1], packed.shape[-1] * 4)


def pack_2bpp_u8(pixels) -> Any:
    """Pack uint8 pixels (0..3) four per byte along the last axis (rl/packed_pixels.py:47-59)."""
    import torch

    if pixels.dtype is not torch.uint8:
        raise ValueError("unpacked_u8 must be uint8")
    if pixels.shape[-1] % 4:
        raise ValueError("last dimension must be divisible by 4")
    q = pixels.reshape(*pixels.shape[:-1], pixels.shape[-1] // 4, 4)
    return q[..., 0] | (q[..., 1] << 2) | (q[..., 2] << 4) | (q[..., 3] << 6)


def s2d_frames(x) -> Any:
    """[B, 1, 72, 80] -> [B, 36, 40, 4]: 2x2 space-to-depth, pixel (y, x) at
    (y // 2, x // 2, (y % 2) * 2 + x % 2) (the layout of
    ``render_pixels_snapshot_packed_scaled_to_torch(..., layout="s2d")``)."""
    b = x.shape[0]
    return x.reshape(b, 36, 2, 40, 2).permute(0, 1, 3, 2, 4).reshape(b, 36, 40, 4)


def s2d_weight(w) -> Any:
    """Conv weight [O, 1, 4, 4] of a stride-2 convolution -> [O, 4, 2, 2] of
    the stride-1 convolution over the 2x2 space-to-depth input that computes
    the same sums: tap (2a + dy, 2b + dx) moves to channel 2 dy + dx at (a, b)."""
    o = w.shape[0]
    return w.reshape(o, 2, 2, 2, 2).permute(0, 2, 4, 1, 3).reshape(o, 4, 2, 2)


def _policy_class():
    import torch
    from torch import nn

    class PixelPolicy(nn.Module):
        def __init__(self, num_actions: int = 9) -> None:
            super().__init__()
            self.conv = nn.Sequential(
                nn.Conv2d(1, 32, 4, stride=2), nn.ReLU(),
                nn.Conv2d(32, 64, 3, stride=2), nn.ReLU(),
                nn.Conv2d(64, 64, 3, stride=1), nn.ReLU(), nn.Flatten())
            with torch.no_grad():
                flat = self.conv(torch.zeros(1, 1, 72, 80)).shape[1]
            self.head = nn.Sequential(nn.Linear(flat, 512), nn.ReLU(), nn.Linear(512, num_actions))

        def forward(self, frames_u8):  # [B, 72, 80] uint8 shades
            return self.forward_scaled(frames_u8.unsqueeze(1).to(self.head[0].weight.dtype) / 3.0)

        def forward_scaled(self, x):  # [B, 1, 72, 80] shades / 3 in the weights' dtype
            # one channel: NCHW and NHWC are the same bytes; channels-last
            # keeps every conv in NHWC (no layout transposes around cuDNN)
            x = x.contiguous(memory_format=torch.channels_last)
            if not x.is_cuda:
                return self.head(self.conv(x))
            # on the GPU each Conv2d + bias + ReLU is one cuDNN call (the
            # unfused module adds the bias and applies the ReLU as two more
            # passes over every activation)
            for conv in (self.conv[0], self.conv[2], self.conv[4]):
                x = torch.ops.aten.cudnn_convolution_relu(x, conv.weight, conv.bias, conv.stride, conv.padding,
                                                         conv.dilation, conv.groups)
            return self._head_nhwc(x)

        def _cached(self, name, src, make):
            # derived weight, rebuilt whenever its source changes (an optimizer
            # step updates the source in place and bumps its version)
            key = (src.data_ptr(), src._version, src.dtype)
            if getattr(self, name + "_key", None) != key:
                setattr(self, name, make(src.detach()))
                setattr(self, name + "_key", key)
            return getattr(self, name)

        def _head_nhwc(self, x):
            # x: the last convolution's output, channels-last. Its features are
            # read in NHWC order (a view, no copy) against the first linear
            # layer's weight with its columns permuted from NCHW to NHWC order:
            # the same sum as flattening NCHW, without the strided copy.
            b, c, hh, ww = x.shape
            lin1, lin2 = self.head[0], self.head[2]
            w1 = self._cached("_w1_nhwc", lin1.weight,
                              lambda w: w.reshape(w.shape[0], c, hh, ww).permute(0, 2, 3, 1).reshape(w.shape[0], -1)
                              .contiguous())
            h = torch.relu(torch.nn.functional.linear(x.permute(0, 2, 3, 1).reshape(b, -1), w1, lin1.bias))
            return torch.nn.functional.linear(h, lin2.weight, lin2.bias)

        def forward_s2d(self, x):  # [B, 36, 40, 4] shades / 3, 2x2 space-to-depth (cell, then (y%2)*2 + x%2)
            # Conv(1->32, k4, s2) over the 72x80 frame is the same sum as a
            # stride-1 k2 convolution over the 4 channels of its 2x2
            # space-to-depth (kernel tap (2a+dy, 2b+dx) -> channel 2dy+dx at
            # (a, b)), which cuDNN runs as an implicit GEMM instead of its
            # one-channel direct engine. GPU only.
            c1 = self.conv[0]
            w = self._cached("_w_s2d", c1.weight,
                             lambda w: s2d_weight(w).contiguous(memory_format=torch.channels_last))
            x = x.permute(0, 3, 1, 2)  # NHWC bytes seen as an NCHW tensor in channels-last order
            x = torch.ops.aten.cudnn_convolution_relu(x, w, c1.bias, (1, 1), (0, 0), (1, 1), 1)
            for conv in (self.conv[2], self.conv[4]):
                x = torch.ops.aten.cudnn_convolution_relu(x, conv.weight, conv.bias, conv.stride, conv.padding,
                                                         conv.dilation, conv.groups)
            return self._head_nhwc(x)

    return PixelPolicy


def make_policy(device, *, num_actions: int = 9, seed: int = 0, dtype=None):
    """Random-init config-5 policy in bf16 on ``device``."""
    import torch

    torch.manual_seed(seed)
    pol = _policy_class()(num_actions).to(device=device, dtype=dtype or torch.bfloat16)
    return pol.to(memory_format=torch.channels_last).eval()


@dataclass
class Rollout:
    actions: list = field(default_factory=list)   # int32 [N] per step (device tensors)
    resets: list = field(default_factory=list)    # bool [N] per step, or None


def run_rollout(backend, policy, steps: int, *, generator=None, chunk: int = 16384,
                reset_cache=None, reset_mask: Callable[[int], Any] | None = None,
                packed_out=None, step_events=None, host_out=None, instr_acc=None) -> Rollout:
    """``steps`` env-steps of render -> policy -> sample -> step.

    ``reset_mask(k)`` (a CUDA bool/uint8 [N] or None) selects envs restored
    from ``reset_cache`` after step k. The policy runs in chunks of ``chunk``
    envs to bound activation memory. ``step_events[k]`` (a pair of CUDA
    events, optional) is recorded around step k's ``step_torch``.
    ``host_out`` (optional pair of pinned host tensors, [2, N, 72, 20] uint8
    and [2, N] int32) receives each step's packed frames and sampled actions,
    copied asynchronously into slot k % 2. ``instr_acc`` (optional int64
    CUDA scalar) accumulates the SM83 instructions each step executed, read
    from the per-env counters around the step and before any restore (a
    restore copies the snapshot's counters). Returns the sampled actions (and
    masks).
    """
    import torch

    n = backend.num_envs
    dev = torch.device("cuda", backend._ordinal)
    packed = packed_out if packed_out is not None else torch.empty((n, 72, 20), dtype=torch.uint8, device=dev)
    # a bf16 policy reads the frames the render writes beside the packed
    # bytes (shade / 3 in bf16: the same values as unpacking and dividing),
    # in the 2x2 space-to-depth layout of its first convolution
    # (this module's bf16 PixelPolicy; any other policy gets the unpacked
    # uint8 frames through its forward)
    wdt = next(policy.parameters()).dtype
    fused = wdt is torch.bfloat16 and hasattr(policy, "forward_s2d")
    scaled = torch.empty((n, 36, 40, 4), dtype=wdt, device=dev) if fused else None
    out = Rollout()
    with torch.no_grad():
        for k in range(steps):
            if scaled is not None:
                backend.render_pixels_snapshot_packed_scaled_to_torch(packed, scaled, layout="s2d")
            else:
                backend.render_pixels_snapshot_packed_to_torch(packed)
            acts = torch.empty(n, dtype=torch.int32, device=dev)
            for lo in range(0, n, chunk):
                hi = min(n, lo + chunk)
                if scaled is not None:
                    logits = policy.forward_s2d(scaled[lo:hi]).float()
                else:
                    logits = policy(unpack_2bpp_u8(packed[lo:hi])).float()
                acts[lo:hi] = torch.multinomial(torch.softmax(logits, dim=-1), 1, generator=generator)[:, 0].to(torch.int32)
            if host_out is not None:
                host_out[0][k % 2].copy_(packed, non_blocking=True)
                host_out[1][k % 2].copy_(acts, non_blocking=True)
            if instr_acc is not None:
                instr_acc -= backend._view("i64")[0].sum()
            if step_events is not None:
                step_events[k][0].record()
            backend.step_torch(acts)
            if step_events is not None:
                step_events[k][1].record()
            if instr_acc is not None:
                instr_acc += backend._view("i64")[0].sum()
            out.actions.append(acts)
            mask = reset_mask(k) if reset_mask is not None else None
            if mask is not None and reset_cache is not None:
                reset_cache.apply_mask_torch(mask)
            out.resets.append(mask)
    return out
