"""Oracle for structured Look attention (test infrastructure only).

Restates ``reference_structured_look_attention``
(layers/triton_structured_look_attention.py:25-54):

    look   = einsum("bqhp,hpqk->bhqk", pose, fields)
    scores = (q.float() @ k.float()^T) * scale;  scores[:, :, 1:, 1:] += look (+ dense)
    out    = (softmax(scores) @ v.float()).to(q.dtype)

Three forms are provided:
  * ``reference_structured_look_attention``: torch-CPU, fp32, the reference's
    own operation sequence (this is also what the CPU baseline times);
  * ``look_attention_np``: numpy, selectable precision (float64 by default),
    general pose/fields/dense form;
  * ``slot_look_attention_np``: numpy, the one-hot-fields case written as a
    gather ``bias[b,h,q,k] = pose[b,q,h,slot(q,k)]`` so large sequences do
    not need an (H, P, Np, Np) tensor.  Mathematically identical to the
    general form with ``fields = onehot(slots)``;
  * ``slot_fields_dense_np``: expands per-slot field values (the compact form
    of the reference model's Look fields) into the general ``(H, P, Np, Np)``
    fields that ``look_attention_np`` takes.
"""

from __future__ import annotations

import numpy as np
import torch

SLOT_NONE = 255


def reference_structured_look_attention(q, k, v, pose, fields, *, scale, dense_bias=None):
    """torch-CPU restatement of layers/triton_structured_look_attention.py:25-54."""
    patches = pose.shape[1]
    if q.shape[-2] != patches + 1:
        raise ValueError("q sequence must contain one CLS token plus pose patches")
    look = torch.einsum("bqhp,hpqk->bhqk", pose, fields)
    scores = (q.float() @ k.float().transpose(-2, -1)) * float(scale)
    scores = scores.clone()
    scores[:, :, 1:, 1:] += look.float()
    if dense_bias is not None:
        expected = (q.shape[0], q.shape[1], patches, patches)
        if tuple(dense_bias.shape) != expected:
            raise ValueError(f"dense_bias must have shape {expected}")
        scores[:, :, 1:, 1:] += dense_bias.float()
    return (scores.softmax(dim=-1) @ v.float()).to(q.dtype)


def _softmax_rows(scores: np.ndarray) -> np.ndarray:
    shifted = scores - scores.max(axis=-1, keepdims=True)
    e = np.exp(shifted)
    return e / e.sum(axis=-1, keepdims=True)


def look_attention_np(q, k, v, pose, fields, *, scale, dense_bias=None, dtype=np.float64, return_lse=False):
    """numpy restatement of the general form; returns float arrays of ``dtype``."""
    q, k, v = (np.asarray(t, dtype=dtype) for t in (q, k, v))
    pose = np.asarray(pose, dtype=dtype)
    fields = np.asarray(fields, dtype=dtype)
    scores = np.einsum("bhqd,bhkd->bhqk", q, k) * dtype(scale)
    scores[:, :, 1:, 1:] += np.einsum("bqhp,hpqk->bhqk", pose, fields)
    if dense_bias is not None:
        scores[:, :, 1:, 1:] += np.asarray(dense_bias, dtype=dtype)
    out = np.einsum("bhqk,bhkd->bhqd", _softmax_rows(scores), v)
    if return_lse:
        m = scores.max(axis=-1)
        lse = m + np.log(np.exp(scores - m[..., None]).sum(axis=-1))
        return out, lse
    return out


def slot_bias_np(pose, slots, *, dtype=np.float64):
    """``bias[b,h,q,k] = pose[b,q,h,slot(q,k)]`` (0 where slot is SLOT_NONE)."""
    pose = np.asarray(pose, dtype=dtype)
    slots = np.asarray(slots)
    batch, patches, heads, n_slots = pose.shape
    padded = np.concatenate([pose, np.zeros((batch, patches, heads, 1), dtype=dtype)], axis=-1)
    index = np.where(slots == SLOT_NONE, n_slots, slots).astype(np.int64)  # (Np, Np)
    per_query = np.transpose(padded, (0, 2, 1, 3))  # (B, H, Np, S + 1)
    index = np.broadcast_to(index[None, None], (batch, heads, patches, patches))
    return np.take_along_axis(per_query, index, axis=-1)  # (B, H, Np, Np)


def slot_look_attention_np(q, k, v, pose, slots, *, scale, dtype=np.float64, return_lse=False):
    """numpy restatement of the one-hot-fields case via a slot gather."""
    q, k, v = (np.asarray(t, dtype=dtype) for t in (q, k, v))
    scores = np.einsum("bhqd,bhkd->bhqk", q, k) * dtype(scale)
    scores[:, :, 1:, 1:] += slot_bias_np(pose, slots, dtype=dtype)
    out = np.einsum("bhqk,bhkd->bhqd", _softmax_rows(scores), v)
    if return_lse:
        m = scores.max(axis=-1)
        lse = m + np.log(np.exp(scores - m[..., None]).sum(axis=-1))
        return out, lse
    return out


def onehot_fields(slots, n_slots: int, heads: int, dtype=np.float32) -> np.ndarray:
    """Dense one-hot ``(H, P, Np, Np)`` fields equal to a slot table."""
    slots = np.asarray(slots)
    patches = slots.shape[0]
    fields = np.zeros((n_slots, patches, patches), dtype=dtype)
    for p in range(n_slots):
        fields[p] = slots == p
    return np.broadcast_to(fields, (heads, n_slots, patches, patches)).copy()


def slot_fields_dense_np(slot_values, slots, dtype=np.float32) -> np.ndarray:
    """Dense ``(H, P, Np, Np)`` fields from per-slot values: ``fields[h, p, q, k] =
    slot_values[h, p, slot(q, k)]``, 0 where the pair has no slot.  This is how
    the reference model's Look bank fields arise (model/deit_tiny_rot_hex_look.py:397-451
    passes them to the attention with a per-head pose): each field plane samples a
    per-head grid at pair geometry, and pairs with the same geometry share a slot."""
    slot_values = np.asarray(slot_values, dtype=dtype)
    slots = np.asarray(slots)
    heads, poses, n_slots = slot_values.shape
    padded = np.concatenate([slot_values, np.zeros((heads, poses, 1), dtype=dtype)], axis=-1)
    index = np.where(slots == SLOT_NONE, n_slots, slots).astype(np.int64)
    return padded[:, :, index]
