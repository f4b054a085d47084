"""SwiGLUDecode on B200 -- iron/operators/swiglu_decode/op.py:13-70.

``W_down @ (SiLU(W_gate @ x) * (W_up @ x))`` for one token, as the same
five-step OperatorSequence IRON builds (one GEMV object reused for the gate and
up projections, then SiLU, ElementwiseMul and the down GEMV), so the runtime
buffers ``in``, ``w_gate``, ``w_up``, ``w_down``, ``left``, ``right``,
``left_swished``, ``intermediate`` and ``out`` are all reachable through
``get_callable().get_buffer(name)``. With the default dispatch the five
kernels run as one CUDA graph per call.
"""

from __future__ import annotations

from ...common.sequence import OperatorSequence
from ..elementwise_mul.op import ElementwiseMul
from ..gemv.op import GEMV
from ..silu.op import SiLU

# IRON sizes its sub-operators from the NPU's shim-DMA budget (16 channels on
# NPU2, halved); the column counts only feed IRON's divisibility checks here.
_N_COLS = 8


class SwiGLUDecode(OperatorSequence):
    """SwiGLU feed-forward for single-token decode (bf16 weights, GEMV layout (M, K))."""

    def __init__(self, embedding_dim, hidden_dim, prio_accuracy=False, context=None, dispatch="auto"):
        self.hidden_dim = hidden_dim
        self.embedding_dim = embedding_dim
        self.prio_accuracy = prio_accuracy
        n_cols = _N_COLS
        gemv_1 = GEMV(M=hidden_dim, K=embedding_dim, num_aie_columns=n_cols, tile_size_input=4,
                      tile_size_output=hidden_dim // n_cols)
        silu = SiLU(size=hidden_dim, num_aie_columns=n_cols, tile_size=hidden_dim // (n_cols * 2))
        eltwise_mul = ElementwiseMul(size=hidden_dim, num_aie_columns=n_cols, tile_size=hidden_dim // n_cols)
        gemv_2 = GEMV(M=embedding_dim, K=hidden_dim, num_aie_columns=n_cols, tile_size_input=1,
                      tile_size_output=embedding_dim // n_cols)
        runlist = [
            (gemv_1, "w_gate", "in", "left"),
            (gemv_1, "w_up", "in", "right"),
            (silu, "left", "left_swished"),
            (eltwise_mul, "left_swished", "right", "intermediate"),
            (gemv_2, "w_down", "intermediate", "out"),
        ]
        super().__init__(name=f"swiglu_decode_e{embedding_dim}_h{hidden_dim}", runlist=runlist,
                         input_args=["in"], output_args=["out"], dispatch=dispatch, context=context)
