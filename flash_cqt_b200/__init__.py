"""B200-native (sm_100a) factored constant-Q transform.

Drop-in for the Flash-CQT API: ``OctCQT``, ``FusedOctCQT``, ``TrainableCQT``,
``SlicedCQT`` and ``Graphed``, all running on hand-written CUDA kernels behind
the C ABI of ``include/flash_cqt_b200.h``; plus ``HostPipeline`` for batches
that live in host memory (copies in both directions overlapped with the
transform).
"""
from .oct_cqt import OctCQT
from .sliced import SlicedCQT
from .graphed import Graphed
from .fused import FusedOctCQT
from .trainable import TrainableCQT
from .hostio import HostPipeline

__all__ = ["OctCQT", "SlicedCQT", "Graphed", "FusedOctCQT", "TrainableCQT", "HostPipeline"]
