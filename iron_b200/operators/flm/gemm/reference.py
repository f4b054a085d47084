"""CPU reference of the flm GEMM (restates iron/operators/flm/gemm/reference.py:8-57):
fp32 accumulation, conversion to bf16, THEN the activation and the clamp."""

import torch

from .design import Epilogue


def apply_epilogue(C, epilogue=Epilogue.NONE, clamp=None):
    e = Epilogue(epilogue)
    if e is Epilogue.GELU:
        C = C * torch.sigmoid(1.702 * C)
    elif e is Epilogue.SILU:
        C = C * torch.sigmoid(C)
    elif e is Epilogue.SIGMOID:
        C = torch.sigmoid(C)
    if clamp is not None:
        C = torch.clamp(C, clamp[0], clamp[1])
    return C


def reference(input_a, input_b, epilogue=Epilogue.NONE, clamp=None):
    C = torch.matmul(input_a.float(), input_b.float()).to(input_a.dtype)
    return apply_epilogue(C, epilogue, clamp)
