"""Multi-scale deformable attention (the MSDeformAttn core of RF-DETR's decoder and encoder) on the
device, forward and backward through ``rfm_msda_forward`` / ``rfm_msda_backward``.

The reference routes this op through a prebuilt Deformable-DETR kernel (kernels_msda_cuda.py,
patches ``fused_msda`` and ``fused_msda_native`` at patches.py:566-635).  This module offers the same
three entry points, on this library's sm_100a kernel:

``ms_deform_attn``        the kernel's native layout: value ``[B, S, M, D]`` (a free view of
                          ``value_proj``'s output) -> ``[B, Q, M * D]``
``deformable_attention``  rf-detr's core contract, value ``[B, M, D, S]`` (``value_by_head``); one
                          layout copy, as the ``fused_msda`` patch makes
``module_forward``        ``MSDeformAttn.forward``'s eager branch with value kept in the native
                          layout (no copy), as the ``fused_msda_native`` patch does

Everything runs in fp32, the precision the replaced ``grid_sample`` path runs at under autocast.
"""

from __future__ import annotations

import ctypes
from typing import Any

import torch
import torch.nn.functional as F

from . import _lib


def _ptr(t: torch.Tensor) -> ctypes.c_void_p:
    return ctypes.c_void_p(t.data_ptr())


def level_start_index(spatial_shapes: torch.Tensor) -> torch.Tensor:
    """Offset of each level's first row in the flattened value sequence."""
    sizes = spatial_shapes[:, 0] * spatial_shapes[:, 1]
    return torch.cat((sizes.new_zeros(1), sizes.cumsum(0)[:-1]))


class _MSDeformAttn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, value, shapes, start, loc, weights):
        batch, seq, heads, dim = value.shape
        queries, levels, points = loc.shape[1], loc.shape[3], loc.shape[4]
        out = torch.empty((batch, queries, heads, dim), dtype=torch.float32, device=value.device)
        stream = ctypes.c_void_p(torch.cuda.current_stream(value.device).cuda_stream)
        _lib.check("rfm_msda_forward", _lib.load().rfm_msda_forward(
            _ptr(value), _ptr(shapes), _ptr(start), _ptr(loc), _ptr(weights), batch, seq, heads, dim, queries,
            levels, points, _ptr(out), stream))
        ctx.save_for_backward(value, shapes, start, loc, weights)
        return out.view(batch, queries, heads * dim)

    @staticmethod
    def backward(ctx, grad_out):
        value, shapes, start, loc, weights = ctx.saved_tensors
        batch, seq, heads, dim = value.shape
        queries, levels, points = loc.shape[1], loc.shape[3], loc.shape[4]
        grad_value = torch.zeros_like(value)
        grad_loc = torch.empty_like(loc)
        grad_w = torch.empty_like(weights)
        g = grad_out.float().contiguous()
        stream = ctypes.c_void_p(torch.cuda.current_stream(value.device).cuda_stream)
        _lib.check("rfm_msda_backward", _lib.load().rfm_msda_backward(
            _ptr(value), _ptr(shapes), _ptr(start), _ptr(loc), _ptr(weights), _ptr(g), batch, seq, heads, dim,
            queries, levels, points, _ptr(grad_value), _ptr(grad_loc), _ptr(grad_w), stream))
        return grad_value, None, None, grad_loc, grad_w


def ms_deform_attn(value: torch.Tensor, spatial_shapes: torch.Tensor, level_start: torch.Tensor | None,
                   sampling_locations: torch.Tensor, attention_weights: torch.Tensor) -> torch.Tensor:
    """Deformable attention in the kernel's layout.

    ``value`` ``[B, S, M, D]``; ``spatial_shapes`` ``[L, 2]`` (H, W) int; ``level_start`` ``[L]`` (or
    None: derived from the shapes); ``sampling_locations`` ``[B, Q, M, L, P, 2]`` in [0, 1];
    ``attention_weights`` ``[B, Q, M, L, P]`` (or ``[B, Q, M, L * P]``).  Returns ``[B, Q, M * D]``
    fp32, differentiable in value, locations and weights.
    """
    if not value.is_cuda:
        raise ValueError("value must be a CUDA tensor (this kernel has no CPU path)")
    if value.dim() != 4 or sampling_locations.dim() != 6:
        raise ValueError("expected value [B, S, M, D] and rank-6 sampling_locations [B, Q, M, L, P, 2]")
    batch, seq, heads, dim = value.shape
    b2, queries, h2, levels, points, two = sampling_locations.shape
    if (b2, h2, two) != (batch, heads, 2) or attention_weights.numel() != batch * queries * heads * levels * points:
        raise ValueError("value, sampling_locations and attention_weights disagree in shape")
    shapes = spatial_shapes.to(device=value.device, dtype=torch.int64).contiguous()
    if shapes.shape != (levels, 2):
        raise ValueError(f"spatial_shapes must be [{levels}, 2]")
    start = level_start_index(shapes) if level_start is None else level_start.to(value.device, torch.int64)
    weights = attention_weights.reshape(batch, queries, heads, levels, points)
    return _MSDeformAttn.apply(value.float().contiguous(), shapes, start.contiguous(),
                               sampling_locations.float().contiguous(), weights.float().contiguous())


def deformable_attention(value_by_head: torch.Tensor, spatial_shapes: torch.Tensor, sampling_locations: torch.Tensor,
                         attention_weights: torch.Tensor, value_spatial_shapes_hw: Any = None) -> torch.Tensor:
    """rf-detr's ``ms_deform_attn_core_pytorch`` contract: value ``[B, M, D, S]`` -> ``[B, Q, M * D]``.
    One layout copy of value (to ``[B, S, M, D]``), as the reference's ``fused_msda`` makes."""
    if sampling_locations.dim() != 6:
        raise ValueError(f"expected rank-6 sampling locations, got shape {tuple(sampling_locations.shape)}")
    value = value_by_head.permute(0, 3, 1, 2)
    return ms_deform_attn(value, spatial_shapes, None, sampling_locations, attention_weights)


def module_forward(module: Any, query: torch.Tensor, reference_points: torch.Tensor, input_flatten: torch.Tensor,
                   input_spatial_shapes: torch.Tensor, input_level_start_index: torch.Tensor,
                   input_padding_mask: torch.Tensor | None = None, input_spatial_shapes_hw: Any = None) -> torch.Tensor:
    """``MSDeformAttn.forward`` (Deformable DETR's module: value/offset/weight projections, softmax over
    levels x points, sampling locations from 2-d or 4-d reference points, output projection) with the
    value kept in the kernel's ``[B, S, M, D]`` layout, a free view of ``value_proj``'s output."""
    batch, len_q, _ = query.shape
    _, len_in, _ = input_flatten.shape
    heads, levels, points = module.n_heads, module.n_levels, module.n_points
    value = module.value_proj(input_flatten)
    if input_padding_mask is not None:
        value = value.masked_fill(input_padding_mask[..., None], 0.0)
    value = value.view(batch, len_in, heads, module.d_model // heads)
    offsets = module.sampling_offsets(query).view(batch, len_q, heads, levels, points, 2)
    weights = module.attention_weights(query).view(batch, len_q, heads, levels * points)
    weights = F.softmax(weights, -1)
    if reference_points.shape[-1] == 2:
        normalizer = torch.stack([input_spatial_shapes[..., 1], input_spatial_shapes[..., 0]], -1)
        locations = reference_points[:, :, None, :, None, :] + offsets / normalizer[None, None, None, :, None, :]
    elif reference_points.shape[-1] == 4:
        locations = (reference_points[:, :, None, :, None, :2]
                     + offsets / points * reference_points[:, :, None, :, None, 2:] * 0.5)
    else:
        raise ValueError(f"last dim of reference_points must be 2 or 4, got {reference_points.shape[-1]}")
    out = ms_deform_attn(value, input_spatial_shapes, input_level_start_index, locations, weights)
    return module.output_proj(out.to(query.dtype))
