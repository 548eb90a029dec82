"""Feature and move-index constants of the network's interface (chessfly/encoding.py:9-18, 85-94).

Board encoding itself (python-chess) belongs to the search, outside this package; the network only
needs the sizes and the from/to square of every policy index.
"""

from __future__ import annotations

import numpy as np

N_BASE = 13 * 64 + 6          # 12 piece planes + en-passant plane, castling rights, halfmove clock, repetition
N_FEATURES = N_BASE + 129     # + the attack planes (read only when ModelConfig.attack_planes is set)
N_MOVES = 64 * 64 + 8 * 3 * 3  # from * 64 + to, plus the underpromotions (file, direction, piece)


def move_squares() -> tuple[np.ndarray, np.ndarray]:
    """From- and to-square of every policy index, in the side-to-move frame (chessfly/encoding.py:85-94):
    index f * 64 + t for f, t < 64; then for each file, direction (left, straight, right) and
    underpromotion piece, a pawn on the 7th rank (48 + file) moving to the 8th (56 + file + direction - 1,
    clipped to the board)."""
    sq = np.arange(4096)
    frm = np.concatenate([sq // 64, np.zeros(72, np.int64)])
    to = np.concatenate([sq % 64, np.zeros(72, np.int64)])
    k = 4096
    for file in range(8):
        for direction in range(3):
            for _piece in range(3):
                frm[k] = 48 + file
                to[k] = 56 + min(max(file + direction - 1, 0), 7)
                k += 1
    return frm.astype(np.int64), to.astype(np.int64)
