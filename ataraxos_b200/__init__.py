"""B200-native StrategoRolloutBuffer: the batched Stratego simulator of Ataraxos.

``StrategoRolloutBuffer`` mirrors the reference's ``_stratego_cuda`` pybind
class and runs every method as hand-written sm_100a CUDA from
``_lib/libstratego_b200.so`` (C ABI: ``include/stratego_b200.h``).
"""

from .buffer import HostStepOutput, StepOutput, StrategoRolloutBuffer, zobrist_table

__all__ = ["StrategoRolloutBuffer", "StepOutput", "HostStepOutput", "zobrist_table"]
