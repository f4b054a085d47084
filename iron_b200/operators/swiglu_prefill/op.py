"""SwiGLUPrefill on B200 -- iron/operators/swiglu_prefill/op.py:13-107.

``W_down @ (SiLU(W_gate @ x) * (W_up @ x))`` over ``seq_len`` tokens, as the same
five-step OperatorSequence IRON builds: one GEMM object reused for the gate and up
projections, then SiLU, ElementwiseMul and the down GEMM. The runtime buffers
``in``, ``w_gate``, ``w_up``, ``w_down``, ``left``, ``right``, ``left_swished``,
``intermediate`` and ``out`` are reachable through ``get_callable().get_buffer(name)``.
``b_col_maj`` stores all three weights as (N, K) (the decode GEMV's layout) instead
of (K, N). The GEMMs run on the tcgen05 tensor cores; with the default dispatch the
five steps (and the weight transposes of the (K, N) layout) run as one CUDA graph.
"""

from __future__ import annotations

from ...common.sequence import OperatorSequence
from ..elementwise_mul.op import ElementwiseMul
from ..gemm.op import GEMM
from ..silu.op import SiLU

# IRON sizes its sub-operators from the NPU's shim-DMA budget (16 channels on NPU2,
# halved); the column count only feeds the operators' divisibility checks here.
_N_COLS = 8


class SwiGLUPrefill(OperatorSequence):
    """SwiGLU feed-forward over a whole prompt (bf16 weights)."""

    def __init__(self, seq_len, embedding_dim, hidden_dim, prio_accuracy=False, b_col_maj=False, context=None,
                 dispatch="auto"):
        self.seq_len = seq_len
        self.hidden_dim = hidden_dim
        self.embedding_dim = embedding_dim
        self.prio_accuracy = prio_accuracy
        self.b_col_maj = b_col_maj
        n_cols = _N_COLS
        # IRON's accuracy knobs select AIE arithmetic; the B200 GEMM always rounds to
        # nearest even from an fp32 accumulator, so they are accepted and validated only
        accuracy = dict(emulate_bf16_mmul_with_bfp16=False, prio_accuracy=True, round_conv_even=True) \
            if prio_accuracy else {}
        gemm_1 = GEMM(M=seq_len, K=embedding_dim, N=hidden_dim, num_aie_columns=n_cols, b_col_maj=b_col_maj,
                      **accuracy)
        self.seq_len_aligned = gemm_1.M
        self.embedding_dim_aligned = gemm_1.K
        self.hidden_dim_aligned = gemm_1.N
        size = self.seq_len_aligned * self.hidden_dim_aligned
        silu = SiLU(size=size, num_aie_columns=n_cols, tile_size=self.hidden_dim_aligned // n_cols)
        eltwise_mul = ElementwiseMul(size=size, num_aie_columns=n_cols, tile_size=self.hidden_dim_aligned // n_cols)
        gemm_2 = GEMM(M=seq_len, K=hidden_dim, N=embedding_dim, num_aie_columns=n_cols, b_col_maj=b_col_maj,
                      **accuracy)
        # GEMM argument order is (input, weight, output); gemm_1 serves gate and up
        runlist = [
            (gemm_1, "in", "w_gate", "left"),
            (gemm_1, "in", "w_up", "right"),
            (silu, "left", "left_swished"),
            (eltwise_mul, "left_swished", "right", "intermediate"),
            (gemm_2, "intermediate", "w_down", "out"),
        ]
        super().__init__(name=f"swiglu_prefill_s{seq_len}_e{embedding_dim}_h{hidden_dim}" + ("_bc" if b_col_maj else ""),
                         runlist=runlist, input_args=["in"], output_args=["out"], dispatch=dispatch, context=context)
