"""Fused learned-address projection on the sm_100a library (``wf_address_projection``).

``LearnedAddressModule.forward_query_key`` (``routing_attention/models/learned_address.py:39-46``)
runs two ``nn.Linear(d_model, d_A)`` projections and ``F.normalize`` on each: six
launches and two passes over the hidden states.  ``address_projection`` stacks the
weights and produces both addresses in one kernel (tcgen05 for bf16/fp16 with fp32
accumulation and normalisation, CUDA cores for fp32), returning views of one
(…, 2·d_A) buffer.  It is forward-only; the module uses it when no gradient is
needed and keeps the PyTorch layers otherwise.
"""

from __future__ import annotations

import torch

from . import _lib


def address_projection(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None, group: int,
                       normalize: bool = True, status: torch.Tensor | None = None) -> torch.Tensor:
    """out[..., n] = x[...] . weight[n] + bias[n], each ``group`` outputs L2-normalised.

    x: (..., d_model) CUDA tensor with unit last stride; weight: (n_out, d_model);
    bias: (n_out,) or None.  Weight and bias are cast to x's dtype.  Returns
    (..., n_out) in x's dtype.
    """
    dev = _lib.require_cuda(x, weight)
    if x.shape[-1] != weight.shape[1]:
        raise ValueError(f"x has {x.shape[-1]} features but weight expects {weight.shape[1]}")
    lead = x.shape[:-1]
    x2 = x.reshape(-1, x.shape[-1])
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    w = weight.to(x.dtype).contiguous()
    b = bias.to(x.dtype).contiguous() if bias is not None else None
    n_out = w.shape[0]
    out = torch.empty(x2.shape[0], n_out, dtype=x.dtype, device=dev)
    lib = _lib.load_library()
    st = _lib.status_arg(dev, status)
    with torch.cuda.device(dev):
        rc = lib.wf_address_projection(
            x2.data_ptr(), _lib.dtype_code(x.dtype), x2.shape[0], x2.shape[1], x2.stride(0), w.data_ptr(),
            b.data_ptr() if b is not None else None, n_out, int(group), 1 if normalize else 0, out.data_ptr(),
            out.stride(0), st, _lib.stream_ptr(dev),
        )
    _lib.check(rc)
    _lib.status_after(dev, status)
    return out.view(*lead, n_out)


class StackedAddressWeights:
    """[W_q; W_k] and [b_q; b_k] rebuilt only when a parameter changes (its version counter)."""

    def __init__(self):
        self._key = None
        self._w = self._b = None

    def get(self, layers) -> tuple[torch.Tensor, torch.Tensor | None]:
        params = [p for l in layers for p in (l.weight, l.bias) if p is not None]
        key = tuple((p.data_ptr(), p._version, p.dtype) for p in params)
        if key != self._key:
            self._w = torch.cat([l.weight.detach() for l in layers], 0)
            has_bias = all(l.bias is not None for l in layers)
            self._b = torch.cat([l.bias.detach() for l in layers], 0) if has_bias else None
            self._key = key
        return self._w, self._b
