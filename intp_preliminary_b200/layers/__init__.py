"""Drop-in module names of the reference's ``layers`` package for the hot path.

``layers/triton_structured_look_attention.py``, ``layers/triton_negative_l1.py`` and
``layers/triton_dense_look_grid.py`` of the reference are replaced by the modules of
the same name here, which re-export the B200 operators with the reference's
function names.
"""
