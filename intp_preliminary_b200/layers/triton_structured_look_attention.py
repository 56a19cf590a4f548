"""Drop-in for the reference's ``layers/triton_structured_look_attention.py``.

Same public name and signature (``structured_look_attention``, :412-424); the
implementation is the sm_100a kernel library, not Triton.  The reference's
explicit oracle ``reference_structured_look_attention`` is test
infrastructure and lives in the repository's ``oracle`` package.
"""

from ..look_attention import LookSlots, structured_look_attention

__all__ = ["LookSlots", "structured_look_attention"]
