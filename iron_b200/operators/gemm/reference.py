"""CPU reference of GEMM (restates iron/operators/gemm/reference.py:7-18): C = A @ B
from the operator's stored layouts."""

import torch


def reference(input_a, input_b, b_col_maj=False, c_col_maj=False):
    B = input_b.T if b_col_maj else input_b
    C = torch.matmul(input_a.float(), B.float()).to(input_a.dtype)
    return C.T if c_col_maj else C
