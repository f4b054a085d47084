"""CPU golden model of GEMV, for ``GEMV.reference`` and compare/reference
sequence dispatch (iron/operators/gemv/reference.py:9-11). Not a fallback: the
operator's callable always runs the CUDA kernel."""

import torch


def dequant_s4g32(codes: torch.Tensor, scales: torch.Tensor) -> torch.Tensor:
    """bf16(q * scale) for the int4g32 layout (low nibble = even k, two's complement)."""
    c = codes.to(torch.int16)
    lo = ((c & 0xF) ^ 8) - 8
    hi = (((c >> 4) & 0xF) ^ 8) - 8
    q = torch.stack([lo, hi], dim=-1).reshape(codes.shape[0], -1).to(torch.float32)
    s = scales.to(torch.float32).repeat_interleave(32, dim=-1)
    return (q * s).to(torch.bfloat16)


def reference(op, *inputs):
    if op.weight_dtype == "int4g32":
        codes, scales, x = inputs
        A = dequant_s4g32(codes, scales)
    else:
        A, x = inputs
    if op.n_vec > 1 or op.num_batches == 1:
        y = x @ A.transpose(-1, -2) if op.n_vec > 1 else A @ x
    else:
        y = torch.einsum("bmk,bk->bm", A.float(), x.float()).to(torch.bfloat16)
    if op.epilogue == "gelu":
        yf = y.float()
        y = (0.5 * yf * (1.0 + torch.tanh(0.7978845608028654 * (yf + 0.044715 * yf**3)))).to(torch.bfloat16)
    return y
