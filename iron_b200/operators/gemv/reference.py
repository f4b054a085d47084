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


def unpack_packed_s4g32(packed: torch.Tensor, M: int, K: int):
    """Inverse of iron_pack_int4g32: packed units -> (codes [M, K/2], scales [M, K/32])."""
    cpt = K // 128
    u = packed.reshape(M // 16, cpt, 1152)
    code = u[:, :, :1024].reshape(M // 16, cpt, 2, 8, 4, 4, 4)  # tile,c,h,gid,tid,j,byte
    code = code.permute(0, 2, 3, 1, 5, 4, 6).reshape(M, K // 2)
    sc = u[:, :, 1024:].reshape(M // 16, cpt, 8, 2, 4, 2).contiguous().view(torch.int16)
    sc = sc.reshape(M // 16, cpt, 8, 2, 4).permute(0, 3, 2, 1, 4).reshape(M, K // 32)
    return code.contiguous(), sc.contiguous().view(torch.bfloat16)


def reference(op, *inputs):
    if op.weight_dtype == "int4g32":
        packed, x = inputs
        codes, scales = unpack_packed_s4g32(packed.reshape(-1), op.M, op.K)
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
