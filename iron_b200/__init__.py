"""iron_b200: IRON's LLM operator hot path on NVIDIA B200 (sm_100a).

``iron_b200.operators`` keeps the constructors and call signatures of
``iron.operators``; the kernels are hand-written CUDA in ``iron_b200/csrc`` behind
the C ABI of ``include/iron_b200.h``, built into ``iron_b200/libiron_b200.so``.
"""

__version__ = "0.1.0"
