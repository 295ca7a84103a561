"""omniASR-LLM decoder attention on B200 (sm_100a): hand-written CUDA behind the ``omniasr_trt.kernels`` API.

``omniasr_b200.kernels`` is the drop-in module; ``omniasr_b200.dropin.install()`` puts it in place of the
reference's ``omniasr_trt.kernels`` when the reference package is importable.
"""

from . import kernels

__all__ = ["kernels"]
