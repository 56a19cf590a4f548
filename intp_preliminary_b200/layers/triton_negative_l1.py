"""Drop-in for the reference's ``layers/triton_negative_l1.py``.

Same public name and signature (``negative_l1_distance``, :233-241); the
implementation is the sm_100a kernel library, not Triton.
"""

from ..negative_l1 import negative_l1_distance

__all__ = ["negative_l1_distance"]
