"""Host restatement of the packed weight layout and the stream-K partition (test helpers).

Packed layout (include/qd_decode.h, csrc/qd_common.cuh): 16 KiB blocks of 128 rows x 64 columns,
row-group-major; inside a block row r is 128 bytes and its 16-byte chunk c sits at c ^ (r & 7).
"""

import numpy as np
import torch


def pack_reference(w: torch.Tensor) -> torch.Tensor:
    """Row-major [n, k] BF16 (n % 128 == 0, k % 64 == 0) -> flat packed BF16 tensor."""
    n, k = w.shape
    assert n % 128 == 0 and k % 64 == 0
    a = w.view(torch.int16).numpy().reshape(n // 128, 128, k // 64, 8, 8)      # g, r, kb, chunk, elem
    a = a.transpose(0, 2, 1, 3, 4).copy()                                     # g, kb, r, chunk, elem
    r = np.arange(128)[:, None]
    c = np.arange(8)[None, :]
    out = np.empty_like(a)
    out[:, :, r, c ^ (r & 7), :] = a[:, :, r, c, :]
    return torch.from_numpy(out.reshape(-1)).view(torch.bfloat16)


def gate_up_interleaved(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """Row-major [2I, k] with 64 gate rows then the 64 matching up rows per 128-row group."""
    inter, k = gate.shape
    return torch.stack([gate.view(inter // 64, 64, k), up.view(inter // 64, 64, k)], 1).reshape(2 * inter, k)


def part_begin(T: int, G: int, c: int) -> int:
    return c * T // G


def part_owner(T: int, G: int, b: int) -> int:
    return ((b + 1) * G - 1) // T
