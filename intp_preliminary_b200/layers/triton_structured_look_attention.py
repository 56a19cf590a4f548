"""Drop-in for the reference's ``layers/triton_structured_look_attention.py``.

Same public name and signature (``structured_look_attention``, :412-424); the
implementation is the sm_100a kernel library, not Triton.  The reference's
explicit oracle ``reference_structured_look_attention`` is test
infrastructure and lives in the repository's ``oracle`` package.

``install_look_bank_hook(SquarePatchDenseGridLook)`` (called once by the
module that replaces the reference's) lets the unchanged reference model's
dense Look-field slices run on the tensor-core kernel in their compact slot
form; see ``intp_preliminary_b200.look_registry``.
"""

from ..look_attention import LookSlotFields, LookSlots, structured_look_attention
from ..look_registry import install_look_bank_hook

__all__ = ["LookSlotFields", "LookSlots", "install_look_bank_hook", "structured_look_attention"]
