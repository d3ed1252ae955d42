"""B200-native packed complex-phase linear layer (hot path of RPFQ-ViT).

Public API:

* :class:`QATLinearComplexPhase` — drop-in for the reference module
  (RPFQ-ViT-main/quant_models/quant_i.py:475-554).
* :class:`VisionAwareQATLinearComplexPhase` — drop-in for the reference's
  token-saliency variant (RPFQ-ViT-main/quant_models/quant_rpfq_vit_vision.py:174-207).
* :class:`PackedPhaseLinear` — the layer over the exporter's packed layout.
* :mod:`rpfq_review_b200.ops` — ``prepack`` (K1 decode), ``gemm`` (K2
  tcgen05 GEMM), ``wide_linear`` (dense or fused decode), ``act_quant``,
  ``vision_act_quant``, ``layernorm``, ``pack_linear`` (GPU packer) and
  ``torch.ops.rpfq.*``.
* :mod:`rpfq_review_b200.packing` — layout, packer, seeded synthetic layers.

The CUDA library (``librpfq_b200.so``, C ABI in ``include/rpfq_b200.h``) is
built in-tree by :func:`rpfq_review_b200.build.build`.
"""

from .packing import PackedLayer, pack_linear, random_packed  # noqa: F401
from .layers import PackedPhaseLinear, QATLinearComplexPhase, VisionAwareQATLinearComplexPhase  # noqa: F401
from . import ops  # noqa: F401

__version__ = "0.1.0"
