"""CPU golden model of Dequant (contract of iron/operators/dequant/reference.py:8-18)."""

import numpy as np
import torch


def reference(payload, tile_size, group_size):
    tile_bytes = tile_size // 2 + 2 * (tile_size // group_size)
    tiles = payload.reshape(-1, tile_bytes).numpy().astype(np.uint8)
    codes = tiles[:, : tile_size // 2]
    q = np.stack([codes & 0xF, codes >> 4], axis=-1).reshape(len(tiles), tile_size)
    sb = tiles[:, tile_size // 2 :].reshape(len(tiles), -1, 2)
    sbits = sb[..., 0].astype(np.uint32) | (sb[..., 1].astype(np.uint32) << 8)
    s = (sbits << 16).view(np.float32)
    out = q.astype(np.float32) * np.repeat(s, group_size, axis=1)
    return torch.from_numpy(out.reshape(-1)).to(torch.bfloat16)
