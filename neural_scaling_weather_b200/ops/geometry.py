"""Window/shift geometry shared by the attention operator and its kernels."""

from __future__ import annotations

from dataclasses import dataclass
from typing import Tuple


@dataclass(frozen=True)
class WindowGeometry:
    """How a (B, T, H, W) token grid is cut into attention windows.

    window:     (wh, ww) window size in tokens.
    shift:      cyclic shift applied by index arithmetic before partitioning: window
                token (r, c) reads grid token ((r + sh) % H, (c + sw) % W), and its
                output is written back to the same grid position.
    mask:       whether the latitude-wrap mask is active (the block is a shifted one).
    mask_shift: the block's latitude shift; rows r_g >= h_global - mask_shift (global,
                rolled coordinates) form the second region.
    row_offset: global row of this rank's first (rolled) row, in tokens.
    h_global:   global number of token rows.
    """

    window: Tuple[int, int]
    shift: Tuple[int, int] = (0, 0)
    mask: bool = False
    mask_shift: int = 0
    row_offset: int = 0
    h_global: int = 0
