"""Drop-in mirror of the reference model API (``w1a1_eagle/model.py``).

Same names, constructor arguments, parameter names and ValueError messages as
the reference; the numerics run in ``libbitdraft.so`` on the GPU.
"""

from __future__ import annotations

import math
from dataclasses import dataclass


@dataclass(frozen=True)
class Geometry:
    """Drafter geometry (``w1a1_eagle/model.py:11-47``), validated the same way."""

    hidden: int = 2560
    intermediate: int = 9216
    heads: int = 32
    kv_heads: int = 8
    head_dim: int = 128
    layers: int = 6
    slots: int = 16
    taps: int = 8
    window: int = 4096
    epsilon: float = 1e-6
    theta: float = 1e7

    def __post_init__(self) -> None:
        sizes = (self.hidden, self.intermediate, self.heads, self.kv_heads, self.head_dim, self.layers, self.slots,
                 self.taps, self.window)
        if any(type(v) is not int or v < 1 for v in sizes):
            raise ValueError("invalid geometry")
        if self.heads % self.kv_heads or self.head_dim % 2:
            raise ValueError("invalid grouped rotary geometry")
        if (not math.isfinite(self.epsilon) or self.epsilon <= 0 or not math.isfinite(self.theta)
                or self.theta <= 0):
            raise ValueError("invalid numerical constants")
