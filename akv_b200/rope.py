"""RoPE cos/sin tables in the layout the reposition kernel reads.

The reference takes the table as an input, ``rotary_emb.cos_sin_cache``
(akv/system/sglang/srt/layers/attention/context_backend.py:392): one row per
position, ``[cos(p * f_0 .. f_{R/2-1}) | sin(...)]``, built by the model's
rotary module in upstream SGLang, which the reference does not vendor.  These
builders are this package's own, written from the published methods:

* ``rope_cos_sin_cache``: plain RoPE (Su et al., 2021), f_i = base^(-2i/R).
* ``yarn_cos_sin_cache``: YaRN (Peng et al., 2023, "YaRN: Efficient Context
  Window Extension of Large Language Models"): per-frequency blend of
  interpolated (f/scale) and extrapolated (f) frequencies with a linear ramp
  between the wavelengths set by ``beta_fast`` and ``beta_slow``, and the
  attention magnitude factor 0.1 ln(scale) + 1 folded into cos and sin.  That
  factor is why cos^2 + sin^2 != 1 and why the kernel divides by it.

Both compute in float32 on the CPU, as a model's rotary module does when it
builds the buffer, and return a float32 tensor ``[max_position, R]``.
"""

from __future__ import annotations

import math

import torch


def _table(inv_freq: torch.Tensor, max_position: int, magnitude: float) -> torch.Tensor:
    t = torch.arange(max_position, dtype=torch.float32)
    freqs = torch.outer(t, inv_freq)
    cos = freqs.cos() * magnitude
    sin = freqs.sin() * magnitude
    return torch.cat((cos, sin), dim=-1).contiguous()


def rope_cos_sin_cache(max_position: int, rotary_dim: int, base: float) -> torch.Tensor:
    inv_freq = 1.0 / (
        base ** (torch.arange(0, rotary_dim, 2, dtype=torch.float32) / rotary_dim)
    )
    return _table(inv_freq, max_position, 1.0)


def _correction_dim(rotary_dim: int, rotations: float, base: float, original_max: int) -> float:
    # Dimension index whose wavelength completes `rotations` turns over the
    # original context (YaRN eq. for the ramp bounds).
    return (rotary_dim * math.log(original_max / (rotations * 2 * math.pi))) / (
        2 * math.log(base)
    )


def yarn_cos_sin_cache(
    max_position: int,
    rotary_dim: int,
    base: float,
    scaling_factor: float,
    original_max_position: int,
    beta_fast: float = 32.0,
    beta_slow: float = 1.0,
    truncate: bool = True,
) -> torch.Tensor:
    """``truncate``: round the ramp's bounds out to whole dimensions (the
    original form of the method); False keeps them fractional, as the
    GPT-OSS checkpoints' rope settings ask ("truncate": false)."""
    half = rotary_dim // 2
    pos_freqs = base ** (torch.arange(0, rotary_dim, 2, dtype=torch.float32) / rotary_dim)
    extrapolation = 1.0 / pos_freqs
    interpolation = 1.0 / (scaling_factor * pos_freqs)
    low = _correction_dim(rotary_dim, beta_fast, base, original_max_position)
    high = _correction_dim(rotary_dim, beta_slow, base, original_max_position)
    if truncate:
        low, high = math.floor(low), math.ceil(high)
    low, high = max(low, 0), min(high, rotary_dim - 1)
    if low == high:
        high += 0.001  # keep the ramp finite
    ramp = ((torch.arange(half, dtype=torch.float32) - low) / (high - low)).clamp(0, 1)
    extrapolate = 1.0 - ramp
    inv_freq = interpolation * (1 - extrapolate) + extrapolation * extrapolate
    magnitude = 0.1 * math.log(scaling_factor) + 1.0 if scaling_factor > 1 else 1.0
    return _table(inv_freq, max_position, magnitude)
