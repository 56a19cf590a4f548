"""CPU port of the reference half6d3r forward (test / baseline infrastructure only).

Runs the reference's CPU algorithm with the weights and geometry tables of a
``ShareViTHalf6d3r``: the tokenizer and Look-bank pose exactly as the model
computes them (they are plain torch ops), the dense Look fields
(36, 12, 195, 195) as the reference builds them once per forward
(layers/square_patch_dense_grid_look.py:357-379), and every layer's attention
through the explicit oracle with those dense fields, which is the reference's
CPU path of ``structured_look_attention`` (layers/triton_structured_look_attention.py:25-54,
:412-418; called from model/deit_tiny_rot_hex_look.py:396-451).
"""

from __future__ import annotations

import math

import numpy as np
import torch

from oracle.look_attention import reference_structured_look_attention


def dense_look_fields(model) -> torch.Tensor:
    """(36, 12, Np, Np) fp32 fields: slot value scattered over the pair table."""
    values = model.slot_fields()                                   # (36, 12, S)
    table = torch.from_numpy(model.look_slots.table.astype(np.int64))
    none = table == 255
    index = torch.where(none, torch.zeros_like(table), table)
    fields = values[:, :, index]                                    # (36, 12, Np, Np)
    fields[:, :, none] = 0.0
    return fields


@torch.no_grad()
def reference_forward_cpu(model, images: torch.Tensor) -> torch.Tensor:
    """Logits of the reference algorithm on CPU (``model.precision`` should be fp32)."""
    tokens, pose = model.embed(images)
    fields = dense_look_fields(model)
    heads = 3
    scale = 1.0 / math.sqrt(64)

    def attend(layer, q, k, v, out):
        sl = slice(heads * layer, heads * (layer + 1))
        return reference_structured_look_attention(q, k, v, pose[:, :, sl], fields[sl], scale=scale)

    feats = model.trunk(tokens, attend)
    return torch.nn.functional.linear(feats[:, 0], model.head.weight, model.head.bias)
