"""bf16 emulation helpers for the oracle (TEST INFRASTRUCTURE ONLY).

The bf16 profile rounds operands to bfloat16 and accumulates in fp32.  To
separate kernel correctness from the precision loss itself, the tests also run
the oracle with the same roundings applied at the same points (weights after
BN folding, activations at every stored bf16 tensor).
"""

from __future__ import annotations

import numpy as np


def round_bf16(x: np.ndarray) -> np.ndarray:
    """Round float32 values to the nearest bfloat16 (ties to even), kept as float32."""
    u = np.ascontiguousarray(x, np.float32).view(np.uint32)
    r = (u + np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))) & np.uint32(0xFFFF0000)
    return r.view(np.float32)
