"""Fast-weight MLP variant (the reference's ``fwpkm/fwmlp.py``).

The MLP variant is not part of the product-key path this package rebuilds.
The module exists so that code importing it at module level
(``modeling_qwen3pkm.py:24``) and testing ``isinstance`` against the class
(``modeling_qwen3pkm.py:736``) keeps working; constructing one raises, as the
PEER variant of ``HashingMemory`` does.
"""
from __future__ import annotations

from torch import nn

from .fwpkm import l2norm  # noqa: F401  (``fwpkm/fwmlp.py:14-17`` exports it too)


class FastWeightMLP(nn.Module):
    """Same constructor signature as ``fwpkm/fwmlp.py:20-36``; not built."""

    def __init__(self, input_dim, output_dim, size, lookahead=0, lookahead_strategy="mean",
                 optimizer_type="sgd", learning_rate=0.1, weight_decay=0.0, loss_type="mse",
                 grad_clip=True, fp32_fw=True):
        super().__init__()
        raise NotImplementedError("the fast-weight MLP variant is not part of the B200 product-key path "
                                  "(fwpkm_variant='pkm' is)")
