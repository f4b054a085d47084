"""CPU golden model of StridedCopy (contract of iron/operators/strided_copy/reference.py:37-75)."""

import numpy as np
import torch


def _pad4(sizes, strides):
    return [1] * (4 - len(sizes)) + list(sizes), [0] * (4 - len(strides)) + list(strides)


def _offsets(sizes, strides, offset, ch):
    sizes, strides = _pad4(sizes, strides)
    per = sizes[3] // ch
    grids = np.meshgrid(*[np.arange(s) for s in sizes[:3] + [per]], indexing="ij")
    out = []
    for c in range(ch):
        flat = np.full(grids[0].shape, offset + c * per * strides[3], dtype=np.int64)
        for g, st in zip(grids, strides):
            flat = flat + g * st
        out.append(flat.reshape(-1))
    return out


def reference(x, in_sizes, in_strides, in_off, out_size, out_sizes, out_strides, out_off, ch=1,
              in_add=0, out_add=0):
    res = torch.zeros(int(out_size), dtype=x.dtype)
    for s, d in zip(_offsets(in_sizes, in_strides, in_off + in_add, ch),
                    _offsets(out_sizes, out_strides, out_off + out_add, ch)):
        res[torch.from_numpy(d)] = x[torch.from_numpy(s)]
    return res
