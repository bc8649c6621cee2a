"""Host-side planning of one SDPA call: compute dtype, broadcast and descriptor.

Given the (validated) operands of a ``scaled_dot_product_attention`` call this
works out what the reference computes implicitly through NumPy broadcasting
(``src/portable_attention/reference.py:139-162``): the broadcast leading shape
of ``Q K^T``, the mask and ``@ V``; which operand strides are 0; and the
grouped-query head mapping (``reference.py:20-53``) expressed as an index
division on the last leading axis instead of a repeat.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from ._lib import (PA_BOOL, PA_F16, PA_F32, PA_F64, PA_MASK_ADD, PA_MASK_BOOL, PA_MASK_NONE,
                   PA_MAX_LEAD, SdpaDesc)

__all__ = ["Plan", "compute_dtype", "plan_call"]

_PA_DTYPE = {np.dtype(np.float16): PA_F16, np.dtype(np.float32): PA_F32,
             np.dtype(np.float64): PA_F64}


def compute_dtype(qd, kd, vd, mask_dtype=None) -> np.dtype:
    """The dtype the device computes in.

    All-fp16 query/key/value stay fp16 on the device (fp32 accumulation inside
    the kernels; an fp16/fp32 additive mask is read as is). Anything else
    computes in ``result_type(q, k, v, float-mask, float32)`` like the fused
    backend (``src/portable_attention/fused.py:178-184``), capped at float64.
    """
    qd, kd, vd = np.dtype(qd), np.dtype(kd), np.dtype(vd)
    half = np.dtype(np.float16)
    float_mask = mask_dtype is not None and np.dtype(mask_dtype) != np.bool_
    if qd == kd == vd == half and (not float_mask or np.dtype(mask_dtype) in (half, np.dtype(np.float32))):
        return half
    parts = [qd, kd, vd] + ([np.dtype(mask_dtype)] if float_mask else [])
    cdt = np.result_type(*parts, np.float32)
    if cdt not in (np.dtype(np.float32), np.dtype(np.float64)):
        cdt = np.dtype(np.float64)
    return cdt


def _lead_strides(shape, out_lead):
    """Element strides of a C-contiguous ``shape`` per ``out_lead`` axis (0 = broadcast)."""
    nl = len(shape) - 2
    dense = [0] * len(shape)
    acc = 1
    for i in range(len(shape) - 1, -1, -1):
        dense[i] = acc
        acc *= shape[i]
    res = []
    n = len(out_lead)
    for i in range(n):
        j = i - (n - nl)
        res.append(dense[j] if j >= 0 and shape[j] != 1 else 0)
    return res


@dataclass
class Plan:
    cdt: np.dtype
    out_lead: tuple
    L: int
    S: int
    E: int
    Ev: int
    group: int
    mask_kind: int
    mask_host_dtype: np.dtype | None
    mask_shape: tuple | None
    desc: SdpaDesc

    @property
    def out_shape(self) -> tuple:
        return (*self.out_lead, self.L, self.Ev)


def plan_call(q_shape, k_shape, v_shape, q_dtype, k_dtype, v_dtype, mask_shape=None,
              mask_dtype=None, is_causal=False, scale=None, group=1) -> Plan:
    """Plan a call on C-contiguous operands of the given shapes and dtypes."""
    q_shape, k_shape, v_shape = tuple(q_shape), tuple(k_shape), tuple(v_shape)
    L, E = q_shape[-2:]
    S, Ev = v_shape[-2:]
    cdt = compute_dtype(q_dtype, k_dtype, v_dtype, mask_dtype)
    q_lead, k_lead, v_lead = q_shape[:-2], k_shape[:-2], v_shape[:-2]
    # Grouped-query: key/value heads broadcast to query heads by index division.
    kx = k_lead[:-1] + (q_lead[-1],) if group > 1 else k_lead
    vx = v_lead[:-1] + (q_lead[-1],) if group > 1 else v_lead
    leads = [q_lead, kx, vx]
    mask_kind, m_host_dt, m_shape = PA_MASK_NONE, None, None
    if mask_shape is not None and not is_causal:
        m_shape = tuple(mask_shape)
        if len(m_shape) < 2:
            m_shape = (1,) * (2 - len(m_shape)) + m_shape
        if m_shape[-2] not in (1, L) or m_shape[-1] not in (1, S):
            raise ValueError(
                f"attn_mask shape {tuple(mask_shape)} is not broadcastable to (*, {L}, {S})")
        leads.append(m_shape[:-2])
        if np.dtype(mask_dtype) == np.bool_:
            mask_kind, m_host_dt = PA_MASK_BOOL, np.dtype(np.uint8)
        else:
            mask_kind = PA_MASK_ADD
            md = np.dtype(mask_dtype)
            if cdt == np.float64 or md not in (np.dtype(np.float16), np.dtype(np.float32)):
                md = np.dtype(np.float64) if cdt == np.float64 else np.dtype(np.float32)
            m_host_dt = md
    out_lead = tuple(np.broadcast_shapes(*leads)) if leads else ()
    if len(out_lead) > PA_MAX_LEAD:
        raise ValueError(f"at most {PA_MAX_LEAD} leading dims are supported, got {len(out_lead)}")

    d = SdpaDesc()
    d.dtype = _PA_DTYPE[cdt]
    d.nlead = len(out_lead)
    for i, n in enumerate(out_lead):
        d.lead[i] = n
    for arr, shape in ((d.q_lead_stride, q_shape), (d.v_lead_stride, v_shape),
                       (d.k_lead_stride, k_shape)):
        for i, s in enumerate(_lead_strides(shape, out_lead)):
            arr[i] = s
    if group > 1:
        # The k/v head axis keeps its real stride: the kernel divides the index.
        ax = len(out_lead) - 1
        d.k_lead_stride[ax] = int(np.prod(k_shape[-2:]))
        d.v_lead_stride[ax] = int(np.prod(v_shape[-2:]))
        d.gqa_axis, d.gqa_group = ax, group
    else:
        d.gqa_axis, d.gqa_group = -1, 1
    d.L, d.S, d.E, d.Ev = L, S, E, Ev
    d.q_row_stride, d.k_row_stride, d.v_row_stride = E, E, Ev
    d.mask_kind = mask_kind
    if mask_kind != PA_MASK_NONE:
        d.mask_dtype = PA_BOOL if mask_kind == PA_MASK_BOOL else _PA_DTYPE[m_host_dt]
        for i, s in enumerate(_lead_strides(m_shape, out_lead)):
            d.m_lead_stride[i] = s
        d.m_row_stride = m_shape[-1] if m_shape[-2] != 1 else 0
        d.m_col_stride = 1 if m_shape[-1] != 1 else 0
    d.is_causal = 1 if is_causal else 0
    d.scale = float(1.0 / np.sqrt(E)) if scale is None else float(scale)
    return Plan(cdt, out_lead, L, S, E, Ev, group, mask_kind, m_host_dt, m_shape, d)
