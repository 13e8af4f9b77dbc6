"""bpdecode_b200 -- the batched constrained-decoding step of bpdecode, rebuilt
for NVIDIA B200 (sm_100a).

Drop-in modules mirroring bpdecode's serving path:

* :mod:`bpdecode_b200.ops` -- ``FsaTensors`` and the per-step dense ops
  (``apply_mask_``, ``advance_state``, ``compute_mask``, ``apply_soft_``);
* :mod:`bpdecode_b200.batch` -- ``ConstraintBatch``, ``GrammarCache``,
  ``MaskCache``;
* :mod:`bpdecode_b200.grammar.device` -- ``PdaTensors``, ``CFGConstraintBatch``
  and the PDA ops;
* :mod:`bpdecode_b200.hf` -- ``GrammarLogitsProcessor`` /
  ``RegexLogitsProcessor``.

All per-step work runs in hand-written CUDA kernels behind the C ABI of
``include/bpdecode_b200.h`` (``libbpdecode_b200.so``, built by
``python -m bpdecode_b200.build``).
"""

from __future__ import annotations

from .tokenizer import Vocabulary

__version__ = "0.1.0"

__all__ = ["Vocabulary", "__version__"]
