"""Host-side E4M3 weight quantisation for the fp8 precision profile.

Weights use the same rowwise scheme as activations (``C3B_K_QUANT_E4M3``):
per output row ``scale = max|w| / 448`` (fp32 division; 1 for an all-zero row),
bytes = E4M3(w / scale) rounded to nearest even.  The conversion is torch's
``float8_e4m3fn`` cast on the CPU after clamping to +-448, which makes it the
saturating conversion the CUDA quantiser uses.
"""

from __future__ import annotations

import numpy as np


def quant_rows_e4m3(w: np.ndarray):
    """[N, K] float -> (uint8 [N, K] E4M3 bytes, float32 [N] scales)."""
    import torch
    w = np.ascontiguousarray(w, np.float32)
    amax = np.max(np.abs(w), axis=1)
    scale = np.where(amax > 0, amax / np.float32(448.0), np.float32(1.0)).astype(np.float32)
    x = np.clip(w / scale[:, None], -448.0, 448.0).astype(np.float32)
    q = torch.from_numpy(x).to(torch.float8_e4m3fn).view(torch.uint8).numpy().copy()
    return q, scale
