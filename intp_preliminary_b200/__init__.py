"""B200-native (sm_100a) SHARE-ViT hot path: structured Look attention and
negative-L1 distance projection behind the reference's Python operator API.

Public operators:
  * ``structured_look_attention`` / ``LookSlots`` / ``LookSlotFields`` (look_attention.py)
  * ``negative_l1_distance`` (negative_l1.py)
The compute runs in ``_lib/libintp_b200.so`` (built by ``build.py``).
"""

from .look_attention import (LookSlotFields, LookSlots, check_device_status, look_attention_backward,
                             look_attention_forward, structured_look_attention)
from .negative_l1 import negative_l1_backward, negative_l1_distance, negative_l1_forward

__all__ = [
    "LookSlotFields",
    "LookSlots",
    "check_device_status",
    "look_attention_backward",
    "look_attention_forward",
    "structured_look_attention",
    "negative_l1_distance",
    "negative_l1_backward",
    "negative_l1_forward",
]
