"""B200-native (sm_100a) SHARE-ViT hot path: structured Look attention and
negative-L1 distance projection behind the reference's Python operator API.

Public operators:
  * ``structured_look_attention`` / ``LookSlots`` / ``LookSlotFields`` (look_attention.py)
  * ``negative_l1_distance`` (negative_l1.py)
  * ``dense_look_grid_sample`` / ``look_sampling_tables`` (dense_look_grid.py)
The compute runs in ``_lib/libintp_b200.so`` (built by ``build.py``).
"""

from .look_attention import (LookSlotFields, LookSlots, check_device_status, look_attention_backward,
                             look_attention_forward, look_probability_score_grad, structured_look_attention)
from .negative_l1 import negative_l1_backward, negative_l1_distance, negative_l1_forward
from .dense_look_grid import (dense_look_grid_backward, dense_look_grid_forward, dense_look_grid_sample,
                              look_sampling_tables)

__all__ = [
    "LookSlotFields",
    "LookSlots",
    "check_device_status",
    "look_attention_backward",
    "look_attention_forward",
    "look_probability_score_grad",
    "structured_look_attention",
    "negative_l1_distance",
    "negative_l1_backward",
    "negative_l1_forward",
    "dense_look_grid_sample",
    "dense_look_grid_forward",
    "dense_look_grid_backward",
    "look_sampling_tables",
]
